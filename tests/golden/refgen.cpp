// refgen — regenerates the inputs and std:: expectations of the reference's
// own GPU tests (Ligo04/lc_parallel_primitive tests/*.cpp) on the host, with
// the same std::mt19937 seed (114521), the same std:: distributions and the
// same std:: algorithms (libstdc++), so that their known answers can pin the
// CPU oracle and the GPU kernels.  Test infrastructure; not part of the
// library.
//
// usage: refgen <case> <out_dir> [n]
// Each array is written as <out_dir>/<name>.<dtype>.bin (little endian).
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <numeric>
#include <random>
#include <string>
#include <utility>
#include <vector>

static std::string g_dir;

template <typename T>
static void dump(const char* name, const char* dt, const std::vector<T>& v) {
    std::string p = g_dir + "/" + name + "." + dt + ".bin";
    FILE* f = std::fopen(p.c_str(), "wb");
    if (!f) { std::perror(p.c_str()); std::exit(2); }
    if (!v.empty()) std::fwrite(v.data(), sizeof(T), v.size(), f);
    std::fclose(f);
}

int main(int argc, char** argv) {
    if (argc < 3) { std::fprintf(stderr, "usage: refgen <case> <out_dir> [n]\n"); return 1; }
    const std::string c = argv[1];
    g_dir = argv[2];
    const uint64_t n = argc > 3 ? std::strtoull(argv[3], nullptr, 10) : 0;

    if (c == "reduce_minmax") {
        // tests/device_reduce_test.cpp:54-62, 118-166: shuffled iota(4096),
        // expected *min_element / *max_element.
        std::vector<int32_t> in(1 << 12);
        for (int i = 0; i < (int)in.size(); i++) in[i] = i;
        std::mt19937 rng(114521);
        std::shuffle(in.begin(), in.end(), rng);
        dump("input", "i32", in);
        dump("min", "i32", std::vector<int32_t>{*std::min_element(in.begin(), in.end())});
        dump("max", "i32", std::vector<int32_t>{*std::max_element(in.begin(), in.end())});
    } else if (c == "sort_float_keys") {
        // tests/device_radix_sort_one_sweep.cpp:61-118: for one size, keys for
        // the ascending and the descending sort drawn alternately from
        // uniform_real_distribution<float>(0,1) with a fresh mt19937(114521).
        std::vector<float> asc(n), desc(n);
        std::mt19937 rng(114521);
        std::uniform_real_distribution<float> dist(0.0f, 1.0f);
        for (uint64_t i = 0; i < n; i++) {
            asc[i] = dist(rng);
            desc[i] = dist(rng);
        }
        dump("asc_in", "f32", asc);
        dump("desc_in", "f32", desc);
        std::sort(asc.begin(), asc.end());
        std::sort(desc.begin(), desc.end(), std::greater<float>());
        dump("asc_expected", "f32", asc);
        dump("desc_expected", "f32", desc);
    } else if (c == "sort_pairs_uint_float") {
        // tests/device_radix_sort_one_sweep.cpp:153-279 (n = 524288): keys are
        // two shuffles of iota, values two runs of uniform(0,1); expected
        // pairs from std::sort by key (keys are unique).
        const int N = n ? (int)n : 524288;
        std::vector<uint32_t> k(N), dk(N);
        std::vector<float> v(N), dv(N);
        std::mt19937 rng(114521);
        std::uniform_real_distribution<float> dist(0.0f, 1.0f);
        for (int i = 0; i < N; i++) { k[i] = (uint32_t)i; dk[i] = (uint32_t)i; }
        std::shuffle(k.begin(), k.end(), rng);
        std::shuffle(dk.begin(), dk.end(), rng);
        for (int i = 0; i < N; i++) { v[i] = dist(rng); dv[i] = dist(rng); }
        dump("keys", "u32", k);
        dump("values", "f32", v);
        dump("desc_keys", "u32", dk);
        dump("desc_values", "f32", dv);
        std::vector<std::pair<uint32_t, float>> p(N), dp(N);
        for (int i = 0; i < N; i++) { p[i] = {k[i], v[i]}; dp[i] = {dk[i], dv[i]}; }
        std::sort(p.begin(), p.end(), [](auto& a, auto& b) { return a.first < b.first; });
        std::sort(dp.begin(), dp.end(), [](auto& a, auto& b) { return a.first > b.first; });
        std::vector<uint32_t> ek(N), edk(N);
        std::vector<float> ev(N), edv(N);
        for (int i = 0; i < N; i++) { ek[i] = p[i].first; ev[i] = p[i].second; edk[i] = dp[i].first; edv[i] = dp[i].second; }
        dump("keys_expected", "u32", ek);
        dump("values_expected", "f32", ev);
        dump("desc_keys_expected", "u32", edk);
        dump("desc_values_expected", "f32", edv);
    } else if (c == "segment_reduce") {
        // tests/device_segment_reduce.cpp:62-125: shuffled iota(1024),
        // segments of 100 items (the last one 24), expected std::accumulate.
        const int N = 1024, per = 100;
        std::vector<int32_t> in(N);
        for (int i = 0; i < N; i++) in[i] = i;
        std::mt19937 rng(114521);
        std::shuffle(in.begin(), in.end(), rng);
        const int S = N / per + 1;
        std::vector<uint32_t> b(S), e(S);
        std::vector<int32_t> sums(S);
        for (int i = 0; i < N; i++)
            if (i % per == 0) {
                b[i / per] = i;
                e[i / per] = std::min(i + per, N);
                sums[i / per] = std::accumulate(in.begin() + i, in.begin() + i + std::min(N - i, per), 0);
            }
        dump("input", "i32", in);
        dump("begin", "u32", b);
        dump("end", "u32", e);
        dump("expected", "i32", sums);
    } else if (c == "fixed_segment_reduce") {
        // tests/device_segment_reduce.cpp:127-176: iota(1024), 32 per segment.
        const int N = 1024, per = 32;
        std::vector<int32_t> in(N);
        for (int i = 0; i < N; i++) in[i] = i;
        std::vector<int32_t> sums(N / per);
        for (int s = 0; s < N / per; s++) sums[s] = std::accumulate(in.begin() + s * per, in.begin() + (s + 1) * per, 0);
        dump("input", "i32", in);
        dump("expected", "i32", sums);
    } else if (c == "reduce_by_key") {
        // tests/device_reduce_test.cpp:54-62, 229-295: shuffled iota(4096),
        // keys i / 100, expected per-run std:: sums and the run count.
        const int N = 1 << 12, per = 100;
        std::vector<int32_t> in(N), keys(N);
        for (int i = 0; i < N; i++) in[i] = i;
        std::mt19937 rng(114521);
        std::shuffle(in.begin(), in.end(), rng);
        for (int i = 0; i < N; i++) keys[i] = i / per;
        const int S = (N + per - 1) / per;
        std::vector<int32_t> sums(S), uk(S);
        for (int s = 0; s < S; s++) {
            sums[s] = std::accumulate(in.begin() + s * per, in.begin() + std::min((s + 1) * per, N), 0);
            uk[s] = s;
        }
        dump("keys", "i32", keys);
        dump("values", "i32", in);
        dump("unique_expected", "i32", uk);
        dump("aggregates_expected", "i32", sums);
        dump("num_runs_expected", "u32", std::vector<uint32_t>{(uint32_t)S});
    } else if (c == "exclusive_sum_by_key") {
        // tests/device_scan_test.cpp:111-167 (one array size n): values all 1,
        // keys i / 100, expected std::exclusive_scan of each segment.
        const int N = (int)n, per = 100;
        std::vector<int32_t> in(N, 1), keys(N), ex(N);
        for (int i = 0; i < N; i++) keys[i] = i / per;
        for (int b = 0; b < N; b += per)
            std::exclusive_scan(in.begin() + b, in.begin() + std::min(b + per, N), ex.begin() + b, 0);
        dump("keys", "i32", keys);
        dump("values", "i32", in);
        dump("expected", "i32", ex);
    } else {
        std::fprintf(stderr, "unknown case %s\n", c.c_str());
        return 1;
    }
    return 0;
}
