// C++ drop-in test: the reference's own device tests (tests/device_reduce_test.cpp,
// device_scan_test.cpp, device_radix_sort_one_sweep.cpp, device_segment_reduce.cpp),
// restated against the B200 build's public headers with the same inputs,
// seeds and std:: expectations.  Exit code 0 = all checks passed.
#include <lcpp/parallel_primitive.h>

#include <algorithm>
#include <cstdio>
#include <functional>
#include <numeric>
#include <random>

using namespace luisa;
using namespace luisa::compute;
using namespace luisa::parallel_primitive;

static int g_failures = 0;
#define EXPECT(cond, ...)                                  \
    do {                                                   \
        if (!(cond)) {                                     \
            ++g_failures;                                  \
            std::printf("FAIL %s:%d ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);                      \
            std::printf("\n");                             \
        }                                                  \
    } while (0)

int main(int argc, char* argv[]) {
    Context context{argv[0]};
    Device device = context.create_device("cuda");
    Stream stream = device.create_stream();

    // ---- device_reduce_test.cpp:66-90 / 118-166 --------------------------------
    {
        DeviceReduce<> reducer;
        reducer.create(device, &stream);
        for (uint loop = 0; loop < 24; ++loop) {
            uint n = (1u << loop) + 1;
            auto d_in = device.create_buffer<uint>(n);
            auto d_out = device.create_buffer<uint>(1);
            std::vector<uint> host(n, 1);
            stream << d_in.copy_from(host.data()) << synchronize();
            size_t tb = DeviceReduce<>::GetTempStorageBytes<uint>(n);
            auto temp = device.create_buffer<uint>(bytes_to_uint_count(tb));
            CommandList cmdlist;
            reducer.Sum(cmdlist, temp.view(), d_in.view(), d_out.view(), n);
            stream << cmdlist.commit() << synchronize();
            std::vector<uint> out(1);
            stream << d_out.copy_to(out.data()) << synchronize();
            EXPECT(out[0] == n, "reduce ones n=%u got %u", n, out[0]);
        }
        const int N = 1 << 12;
        std::vector<int32> input(N);
        std::iota(input.begin(), input.end(), 0);
        std::mt19937 rng(114521);
        std::shuffle(input.begin(), input.end(), rng);
        auto d_in = device.create_buffer<int32>(N);
        auto d_out = device.create_buffer<int32>(1);
        stream << d_in.copy_from(input.data()) << synchronize();
        auto temp = device.create_buffer<uint>(bytes_to_uint_count(DeviceReduce<>::GetTempStorageBytes<int32>(N)));
        std::vector<int32> r(1);
        CommandList cmdlist;
        reducer.Min(cmdlist, temp.view(), d_in.view(), d_out.view(), d_in.size());
        stream << cmdlist.commit() << synchronize() << d_out.copy_to(r.data()) << synchronize();
        EXPECT(r[0] == *std::min_element(input.begin(), input.end()), "reduce min %d", r[0]);
        reducer.Max(cmdlist, temp.view(), d_in.view(), d_out.view(), d_in.size());
        stream << cmdlist.commit() << synchronize() << d_out.copy_to(r.data()) << synchronize();
        EXPECT(r[0] == *std::max_element(input.begin(), input.end()), "reduce max %d", r[0]);
    }

    // ---- device_scan_test.cpp:67-108 ------------------------------------------
    {
        using ScannerT = DeviceScan<256, 32, 4>;
        ScannerT scanner;
        scanner.create(device, &stream);
        CommandList cmdlist;
        for (int i = 0; i < 24; i++) {
            const uint n = 1u << i;
            std::vector<uint> input(n, 1);
            auto in = device.create_buffer<uint>(n);
            auto ex = device.create_buffer<uint>(n);
            auto inc = device.create_buffer<uint>(n);
            stream << in.copy_from(input.data()) << synchronize();
            auto temp = device.create_buffer<uint>(bytes_to_uint_count(ScannerT::GetTempStorageBytes<uint>(n)));
            scanner.ExclusiveSum(cmdlist, temp.view(), in.view(), ex.view(), in.size());
            stream << cmdlist.commit() << synchronize();
            scanner.InclusiveSum(cmdlist, temp.view(), in.view(), inc.view(), in.size());
            stream << cmdlist.commit() << synchronize();
            std::vector<uint> er(n), ir(n), ee(n), ie(n);
            stream << ex.copy_to(er.data()) << inc.copy_to(ir.data()) << synchronize();
            std::exclusive_scan(input.begin(), input.end(), ee.begin(), 0u);
            std::inclusive_scan(input.begin(), input.end(), ie.begin());
            EXPECT(er == ee && ir == ie, "scan failed for size 2^%d", i);
        }
    }

    // ---- device_radix_sort_one_sweep.cpp:61-151, 153-279 -----------------------
    {
        using SorterT = DeviceRadixSort<128, 32, 4>;
        SorterT sorter;
        sorter.create(device, &stream);
        CommandList cmdlist;
        for (uint loop = 5; loop < 25; ++loop) {
            uint n = 1u << loop;
            std::vector<float> a(n), d(n);
            std::mt19937 rng(114521);
            std::uniform_real_distribution<float> dist(0.0f, 1.0f);
            for (uint i = 0; i < n; i++) { a[i] = dist(rng); d[i] = dist(rng); }
            auto ain = device.create_buffer<float>(n), aout = device.create_buffer<float>(n);
            auto din = device.create_buffer<float>(n), dout = device.create_buffer<float>(n);
            stream << ain.copy_from(a.data()) << din.copy_from(d.data()) << synchronize();
            auto temp = device.create_buffer<uint>(bytes_to_uint_count(SorterT::GetSortKeysTempStorageBytes<float>(n)));
            sorter.SortKeys<float>(cmdlist, temp.view(), ain.view(), aout.view(), ain.size());
            sorter.SortKeysDescending<float>(cmdlist, temp.view(), din.view(), dout.view(), din.size());
            stream << cmdlist.commit() << synchronize();
            std::vector<float> ar(n), dr(n);
            stream << aout.copy_to(ar.data()) << dout.copy_to(dr.data()) << synchronize();
            std::sort(a.begin(), a.end());
            std::sort(d.begin(), d.end(), std::greater<float>());
            EXPECT(ar == a, "float asc n=%u", n);
            EXPECT(dr == d, "float desc n=%u", n);
        }
        DeviceRadixSort<> s2;
        s2.create(device, &stream);
        for (uint loop = 0; loop < 24; ++loop) {
            uint n = 1u << loop;
            std::vector<uint> keys(n);
            for (uint i = 0; i < n; ++i) keys[i] = n - i - 1;
            auto kin = device.create_buffer<uint>(n), kout = device.create_buffer<uint>(n);
            stream << kin.copy_from(keys.data()) << synchronize();
            auto temp = device.create_buffer<uint>(bytes_to_uint_count(DeviceRadixSort<>::GetSortKeysTempStorageBytes<uint>(n)));
            CommandList cl;
            s2.SortKeys(cl, temp.view(), kin.view(), kout.view(), n);
            stream << cl.commit() << synchronize();
            std::vector<uint> r(n);
            stream << kout.copy_to(r.data()) << synchronize();
            std::sort(keys.begin(), keys.end());
            EXPECT(r == keys, "uint reversed n=%u", n);
        }
        const int N = 524288;
        std::vector<uint> k(N), dk(N);
        std::vector<float> v(N), dv(N);
        std::mt19937 rng(114521);
        std::uniform_real_distribution<float> dist(0.0f, 1.0f);
        for (int i = 0; i < N; i++) { k[i] = i; dk[i] = i; }
        std::shuffle(k.begin(), k.end(), rng);
        std::shuffle(dk.begin(), dk.end(), rng);
        for (int i = 0; i < N; i++) { v[i] = dist(rng); dv[i] = dist(rng); }
        std::vector<std::pair<uint, float>> p(N), dp(N);
        for (int i = 0; i < N; i++) { p[i] = {k[i], v[i]}; dp[i] = {dk[i], dv[i]}; }
        auto kb = device.create_buffer<uint>(N), ko = device.create_buffer<uint>(N);
        auto vb = device.create_buffer<float>(N), vo = device.create_buffer<float>(N);
        auto dkb = device.create_buffer<uint>(N), dko = device.create_buffer<uint>(N);
        auto dvb = device.create_buffer<float>(N), dvo = device.create_buffer<float>(N);
        stream << kb.copy_from(k.data()) << vb.copy_from(v.data()) << dkb.copy_from(dk.data())
               << dvb.copy_from(dv.data()) << synchronize();
        auto temp = device.create_buffer<uint>(bytes_to_uint_count(SorterT::GetSortPairsTempStorageBytes<uint, float>(N)));
        sorter.SortPairs<uint, float>(cmdlist, temp.view(), kb.view(), ko.view(), vb.view(), vo.view(), kb.size());
        stream << cmdlist.commit() << synchronize();
        sorter.SortPairsDescending<uint, float>(cmdlist, temp.view(), dkb.view(), dko.view(), dvb.view(), dvo.view(),
                                                dkb.size());
        stream << cmdlist.commit() << synchronize();
        std::vector<uint> rk(N), rdk(N);
        std::vector<float> rv(N), rdv(N);
        stream << ko.copy_to(rk.data()) << vo.copy_to(rv.data()) << dko.copy_to(rdk.data())
               << dvo.copy_to(rdv.data()) << synchronize();
        std::sort(p.begin(), p.end(), [](auto& a, auto& b) { return a.first < b.first; });
        std::sort(dp.begin(), dp.end(), [](auto& a, auto& b) { return a.first > b.first; });
        bool ok = true, dok = true;
        for (int i = 0; i < N; i++) {
            ok &= rk[i] == p[i].first && rv[i] == p[i].second;
            dok &= rdk[i] == dp[i].first && rdv[i] == dp[i].second;
        }
        EXPECT(ok, "pairs ascending");
        EXPECT(dok, "pairs descending");
    }

    // ---- device_segment_reduce.cpp:62-176 --------------------------------------
    {
        DeviceSegmentReduce<> reducer;
        reducer.create(device, &stream);
        CommandList cmdlist;
        const int N = 1024, per = 100;
        std::vector<int32> input(N);
        std::iota(input.begin(), input.end(), 0);
        std::mt19937 rng(114521);
        std::shuffle(input.begin(), input.end(), rng);
        const int S = N / per + 1;
        std::vector<uint> b(S), e(S);
        for (int i = 0; i < N; i++)
            if (i % per == 0) { b[i / per] = i; e[i / per] = std::min(i + per, N); }
        auto in = device.create_buffer<int32>(N);
        auto out = device.create_buffer<int32>(S);
        auto bb = device.create_buffer<uint>(S), eb = device.create_buffer<uint>(S);
        stream << in.copy_from(input.data()) << bb.copy_from(b.data()) << eb.copy_from(e.data()) << synchronize();
        auto temp = device.create_buffer<uint>(
            std::max<size_t>(1, bytes_to_uint_count(DeviceSegmentReduce<>::GetTempStorageBytes<int32>(N))));
        reducer.Sum(cmdlist, temp.view(), in.view(), out.view(), S, bb.view(), eb.view());
        stream << cmdlist.commit() << synchronize();
        std::vector<int32> r(S);
        stream << out.copy_to(r.data()) << synchronize();
        for (int s = 0; s < S; s++) {
            int want = std::accumulate(input.begin() + b[s], input.begin() + e[s], 0);
            EXPECT(r[s] == want, "segment %d got %d want %d", s, r[s], want);
        }
        // fixed size: 32 segments of 32 over iota(1024)
        std::vector<int32> iota(N);
        std::iota(iota.begin(), iota.end(), 0);
        auto in2 = device.create_buffer<int32>(N);
        auto out2 = device.create_buffer<int32>(32);
        stream << in2.copy_from(iota.data()) << synchronize();
        reducer.Sum(cmdlist, temp.view(), in2.view(), out2.view(), 32u, 32u);
        stream << cmdlist.commit() << synchronize();
        std::vector<int32> r2(32);
        stream << out2.copy_to(r2.data()) << synchronize();
        for (int s = 0; s < 32; s++) {
            int want = std::accumulate(iota.begin() + s * 32, iota.begin() + (s + 1) * 32, 0);
            EXPECT(r2[s] == want, "fixed segment %d", s);
        }
    }

    // ---- device_reduce_test.cpp:168-220 / device_segment_reduce.cpp:179-293: Arg* --
    {
        const int N = 1 << 12;
        std::vector<int32> input(N);
        std::iota(input.begin(), input.end(), 0);
        std::mt19937 rng(114521);
        std::shuffle(input.begin(), input.end(), rng);
        DeviceReduce<> reducer;
        reducer.create(device, &stream);
        auto in = device.create_buffer<int32>(N);
        auto out = device.create_buffer<int32>(1);
        auto idx = device.create_buffer<uint>(1);
        stream << in.copy_from(input.data()) << synchronize();
        auto temp = device.create_buffer<uint>(bytes_to_uint_count(DeviceReduce<>::GetArgTempStorageBytes<int32>(N)));
        CommandList cmdlist;
        std::vector<uint> ri(1);
        reducer.ArgMin(cmdlist, temp.view(), in.view(), out.view(), idx.view(), in.size());
        stream << cmdlist.commit() << synchronize() << idx.copy_to(ri.data()) << synchronize();
        EXPECT(ri[0] == (uint)(std::min_element(input.begin(), input.end()) - input.begin()), "argmin %u", ri[0]);
        reducer.ArgMax(cmdlist, temp.view(), in.view(), out.view(), idx.view(), in.size());
        stream << cmdlist.commit() << synchronize() << idx.copy_to(ri.data()) << synchronize();
        EXPECT(ri[0] == (uint)(std::max_element(input.begin(), input.end()) - input.begin()), "argmax %u", ri[0]);

        const int per = 100, S = N / per + 1;
        std::vector<uint> b(S), e(S);
        for (int s = 0; s < S; s++) { b[s] = s * per; e[s] = std::min(s * per + per, N); }
        DeviceSegmentReduce<> sr;
        sr.create(device, &stream);
        auto sv = device.create_buffer<int32>(S);
        auto si = device.create_buffer<uint>(S);
        auto bb = device.create_buffer<uint>(S), eb = device.create_buffer<uint>(S);
        stream << bb.copy_from(b.data()) << eb.copy_from(e.data()) << synchronize();
        std::vector<int32> rv(S);
        std::vector<uint> rix(S);
        sr.ArgMax(cmdlist, temp.view(), in.view(), sv.view(), si.view(), S, bb.view(), eb.view());
        stream << cmdlist.commit() << synchronize() << sv.copy_to(rv.data()) << si.copy_to(rix.data()) << synchronize();
        for (int s = 0; s < S; s++) {
            auto m = std::max_element(input.begin() + b[s], input.begin() + e[s]);
            EXPECT(rv[s] == *m && rix[s] == (uint)(m - input.begin() - b[s]), "segment argmax %d", s);
        }
        sr.ArgMin(cmdlist, temp.view(), in.view(), sv.view(), si.view(), S, bb.view(), eb.view());
        stream << cmdlist.commit() << synchronize() << sv.copy_to(rv.data()) << si.copy_to(rix.data()) << synchronize();
        for (int s = 0; s < S; s++) {
            auto m = std::min_element(input.begin() + b[s], input.begin() + e[s]);
            EXPECT(rv[s] == *m && rix[s] == (uint)(m - input.begin() - b[s]), "segment argmin %d", s);
        }
    }

    // ---- device_reduce_test.cpp:92-116 (TransformReduce: max of squares) ----------
    {
        const int N = 1 << 12;
        std::vector<int32> input(N);
        std::iota(input.begin(), input.end(), 0);
        std::mt19937 rng(114521);
        std::shuffle(input.begin(), input.end(), rng);
        DeviceReduce<> reducer;
        reducer.create(device, &stream);
        auto in = device.create_buffer<int32>(N);
        auto out = device.create_buffer<int32>(1);
        stream << in.copy_from(input.data()) << synchronize();
        auto temp = device.create_buffer<uint>(bytes_to_uint_count(DeviceReduce<>::GetTempStorageBytes<int32>(N)));
        CommandList cmdlist;
        reducer.TransformReduce(cmdlist, temp.view(), in.view(), out.view(), in.size(), MaxOp{}, SquareOp{}, 0);
        std::vector<int32> r(1);
        stream << cmdlist.commit() << synchronize() << out.copy_to(r.data()) << synchronize();
        EXPECT(r[0] == (N - 1) * (N - 1), "transform reduce %d", r[0]);
    }

    // ---- device_scan_test.cpp:111-167 (ExclusiveSumByKey) / device_reduce_test.cpp:229-295 --
    {
        DeviceScan<> scanner;
        scanner.create(device, &stream);
        for (int i = 5; i < 24; i += 6) {
            const uint n = 1u << i;
            const int per = 100;
            std::vector<int32> ones(n, 1), keys(n);
            for (uint j = 0; j < n; j++) keys[j] = (int32)(j / per);
            auto kb = device.create_buffer<int32>(n), vb = device.create_buffer<int32>(n), ob = device.create_buffer<int32>(n);
            stream << kb.copy_from(keys.data()) << vb.copy_from(ones.data()) << synchronize();
            auto temp = device.create_buffer<uint>(
                bytes_to_uint_count(DeviceScan<>::GetScanByKeyTempStorageBytes<int32, int32>(n)));
            CommandList cmdlist;
            scanner.ExclusiveSumByKey(cmdlist, temp.view(), kb.view(), vb.view(), ob.view(), kb.size());
            std::vector<int32> res(n);
            stream << cmdlist.commit() << synchronize() << ob.copy_to(res.data()) << synchronize();
            int bad = 0;
            for (uint j = 0; j < n; j++) bad += res[j] != (int32)(j % per);
            EXPECT(bad == 0, "exclusive_sum_by_key n=%u: %d wrong", n, bad);
        }
        const int N = 1 << 12, per = 100, S = (N + per - 1) / per;
        std::vector<int32> input(N), keys(N);
        std::iota(input.begin(), input.end(), 0);
        std::mt19937 rng(114521);
        std::shuffle(input.begin(), input.end(), rng);
        for (int j = 0; j < N; j++) keys[j] = j / per;
        DeviceReduce<> reducer;
        reducer.create(device, &stream);
        auto kb = device.create_buffer<int32>(N), vb = device.create_buffer<int32>(N);
        auto ub = device.create_buffer<int32>(S), ab = device.create_buffer<int32>(S);
        auto rb = device.create_buffer<uint>(1);
        stream << kb.copy_from(keys.data()) << vb.copy_from(input.data()) << synchronize();
        auto temp = device.create_buffer<uint>(
            bytes_to_uint_count(DeviceReduce<>::GetReduceByKeyTempStorageBytes<int32, int32>(N)));
        CommandList cmdlist;
        reducer.ReduceByKey(cmdlist, temp.view(), kb.view(), vb.view(), ub.view(), ab.view(), rb.view(), SumOp{},
                            kb.size());
        std::vector<int32> uk(S), agg(S);
        std::vector<uint> runs(1);
        stream << cmdlist.commit() << synchronize() << ub.copy_to(uk.data()) << ab.copy_to(agg.data())
               << rb.copy_to(runs.data()) << synchronize();
        EXPECT(runs[0] == (uint)S, "reduce_by_key runs %u", runs[0]);
        for (int s = 0; s < S; s++) {
            int want = std::accumulate(input.begin() + s * per, input.begin() + std::min((s + 1) * per, N), 0);
            EXPECT(agg[s] == want && uk[s] == s, "reduce_by_key run %d", s);
        }
    }

    // ---- MultiDevice (multi-GPU extension) on a 1-rank NCCL communicator -----
    {
        std::vector<char> uid(lcpp_mg_unique_id_bytes());
        void* comm = nullptr;
        if (lcpp_mg_get_unique_id(uid.data()) == LCPP_OK && lcpp_mg_comm_init_rank(&comm, 1, uid.data(), 0) == LCPP_OK) {
            MultiDevice mg;
            mg.create(device, comm, &stream);
            const uint n = 300007;
            std::vector<uint64_t> keys(n);
            std::vector<uint> vals(n);
            std::mt19937_64 rng(114521);
            for (uint j = 0; j < n; j++) { keys[j] = rng() & 0xFFFFFull; vals[j] = j; }
            auto kin = device.create_buffer<uint64_t>(n), kout = device.create_buffer<uint64_t>(n);
            auto vin = device.create_buffer<uint>(n), vout = device.create_buffer<uint>(n);
            stream << kin.copy_from(keys.data()) << vin.copy_from(vals.data()) << synchronize();
            auto temp = device.create_buffer<uint>(
                bytes_to_uint_count(MultiDevice::GetSortPairsTempStorageBytes<uint64_t, uint>(n, n, 1)));
            uint64_t n_out = 0;
            CommandList cmdlist;
            mg.SortPairs(cmdlist, temp.view(), kin.view(), kout.view(), vin.view(), vout.view(), n, n, &n_out);
            std::vector<uint64_t> ko(n);
            std::vector<uint> vo(n);
            stream << cmdlist.commit() << synchronize() << kout.copy_to(ko.data()) << vout.copy_to(vo.data())
                   << synchronize();
            std::vector<uint> idx(n);
            std::iota(idx.begin(), idx.end(), 0u);
            std::stable_sort(idx.begin(), idx.end(), [&](uint a, uint b) { return keys[a] < keys[b]; });
            int bad = 0;
            for (uint j = 0; j < n; j++) bad += ko[j] != keys[idx[j]] || vo[j] != idx[j];
            EXPECT(n_out == n && bad == 0, "MultiDevice SortPairs: n_out %llu, %d wrong", (unsigned long long)n_out, bad);
            auto sin = device.create_buffer<uint>(n), sout = device.create_buffer<uint>(n), red = device.create_buffer<uint>(1);
            stream << sin.copy_from(vals.data()) << synchronize();
            auto st = device.create_buffer<uint>(bytes_to_uint_count(
                std::max(MultiDevice::GetScanTempStorageBytes<uint>(n, 1), MultiDevice::GetReduceTempStorageBytes<uint>(n))));
            mg.ExclusiveSum(cmdlist, st.view(), sin.view(), sout.view(), n);
            stream << cmdlist.commit() << synchronize();
            mg.Max(cmdlist, st.view(), sin.view(), red.view(), n);
            std::vector<uint> so(n), rmax(1);
            stream << cmdlist.commit() << synchronize() << sout.copy_to(so.data()) << red.copy_to(rmax.data())
                   << synchronize();
            bad = 0;
            uint acc = 0;
            for (uint j = 0; j < n; j++) { bad += so[j] != acc; acc += vals[j]; }
            EXPECT(bad == 0 && rmax[0] == n - 1, "MultiDevice ExclusiveSum/Max: %d wrong, max %u", bad, rmax[0]);
            lcpp_mg_comm_destroy(comm);
        } else {
            EXPECT(false, "could not make a 1-rank NCCL communicator");
        }
    }

    EXPECT(stream.last_status() == 0, "stream status %d", stream.last_status());
    std::printf("%s: %d failure(s)\n", g_failures ? "FAILED" : "OK", g_failures);
    return g_failures ? 1 : 0;
}
