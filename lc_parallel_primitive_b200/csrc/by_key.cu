// ScanByKey and ReduceByKey for sm_100a: single-pass segmented scan with
// decoupled look-back over (count, value) pairs.
//
// Reference behaviour followed:
//  * DeviceScan::ExclusiveScanByKey / InclusiveScanByKey
//    (src/lcpp/device/device_scan.h:206-300) and ScanByKeyModule
//    (src/lcpp/device/details/scan_by_key.h): a segment starts at item 0 and
//    wherever keys[i] != keys[i-1]; the pair operator is ScanBySegmentOp
//    (src/lcpp/common/thread_operators.h:107-127); AddInitToScan gives
//    exclusive out[i] = init at a segment head, scan_op(prefix, init) elsewhere.
//    Inclusive out[i] = scan_op(v[head..i], init) at every item.  (The
//    reference's AddInitToScan also replaces an inclusive head's own value by
//    init, which drops v[head] from that item only while later items of the
//    segment include it; that inconsistency is not reproduced.)
//  * DeviceReduce::ReduceByKey (src/lcpp/device/device_reduce.h:277-325) and
//    ReduceByKeyModule (src/lcpp/device/details/reduce_by_key.h): one output
//    per run of equal consecutive keys, unique_out[r] = the key of the run's
//    last item, aggregates_out[r] = reduce_op over the run, num_runs_out[0] =
//    number of runs (0 for empty input).
//
// B200 design:
//  * Tiles of 512 threads x ITEMS items (8192 items for 4-byte keys and
//    values).  Keys and values are read with coalesced 128-bit striped loads
//    into shared memory and read back blocked (each thread ITEMS consecutive
//    items) through an XOR swizzle that makes both directions free of bank
//    conflicts.
//  * Per thread a sequential pair scan; per warp a shuffle scan of pairs; one
//    16-entry scan of warp totals; warp 0 resolves the tile prefix by a
//    warp-wide look-back (32 predecessors per poll, ordered reduction because
//    the pair operator does not commute).
//  * Descriptors: for 4-byte values and n < 2^30 one 64-bit word per tile
//    {status | count | value} with relaxed accesses (no fences); otherwise
//    two or three relaxed words per tile, each carrying the status beside one
//    part of the pair, accepted when all statuses match.  Every wait is
//    bounded by g_spin_limit.
//  * Outputs are staged in shared memory and written coalesced: the scanned
//    values back through the same swizzle, the runs of ReduceByKey compacted
//    to a dense range per tile.
#include "bulk.cuh"
#include "common.cuh"

namespace lcpp {

constexpr int BK_THREADS = 512;
constexpr int BK_WARPS = BK_THREADS / 32;
constexpr size_t BK_HDR = 256;

enum BkMode { BK_SCAN_EXCL = 0, BK_SCAN_INCL = 1, BK_REDUCE = 2 };

// (count, value): count = number of segment heads covered, value = the
// reduction since the last head.
template <typename T>
struct alignas(sizeof(T) == 8 ? 16 : 8) KPair {
    uint32_t count;
    T value;
};

template <typename Op, typename T>
__device__ __forceinline__ KPair<T> kcombine(const KPair<T>& a, const KPair<T>& b) {
    KPair<T> r;
    r.count = a.count + b.count;
    r.value = b.count ? b.value : Op::template apply<T>(a.value, b.value);
    return r;
}

template <typename Op, typename T>
__device__ __forceinline__ KPair<T> kidentity() {
    KPair<T> r;
    r.count = 0;
    r.value = Op::template identity<T>();
    return r;
}

template <typename T>
__device__ __forceinline__ KPair<T> kshfl_up(const KPair<T>& p, int o) {
    KPair<T> r;
    r.count = __shfl_up_sync(0xffffffffu, p.count, o);
    r.value = __shfl_up_sync(0xffffffffu, p.value, o);
    return r;
}
template <typename T>
__device__ __forceinline__ KPair<T> kshfl_down(const KPair<T>& p, int o) {
    KPair<T> r;
    r.count = __shfl_down_sync(0xffffffffu, p.count, o);
    r.value = __shfl_down_sync(0xffffffffu, p.value, o);
    return r;
}
template <typename T>
__device__ __forceinline__ KPair<T> kshfl(const KPair<T>& p, int src) {
    KPair<T> r;
    r.count = __shfl_sync(0xffffffffu, p.count, src);
    r.value = __shfl_sync(0xffffffffu, p.value, src);
    return r;
}

// Two descriptor forms, both written and read with relaxed device-scope
// accesses only (no fences).  Packed (4-byte values, n < 2^30): one 64-bit
// word per tile {status:2 | count:30 | value:32}.  Split (otherwise): WPT
// 64-bit words per tile, {status:32 | count:32}, {status:32 | value bits
// 0..31} and, for 8-byte values, {status:32 | value bits 32..63}.  Each
// status is written once per tile with one pair, so when every word of a
// tile shows the same status the words belong to the same pair; a reader
// that sees different statuses (a write in between) polls the tile again.
template <typename T>
struct BkDesc {
    uint64_t* packed;  // non-null: packed form
    uint64_t* split;   // otherwise: [tiles][WPT]
    static constexpr int WPT = sizeof(T) == 8 ? 3 : 2;
};

struct BkRaw {
    uint64_t w[3];
};

template <typename T>
__device__ __forceinline__ uint64_t bk_pack(uint32_t st, const KPair<T>& p) {
    uint32_t b;
    memcpy(&b, &p.value, 4);
    return (uint64_t)st << 62 | (uint64_t)(p.count & 0x3fffffffu) << 32 | b;
}
template <typename T>
__device__ __forceinline__ KPair<T> bk_unpack(uint64_t w) {
    KPair<T> p;
    p.count = (uint32_t)(w >> 32) & 0x3fffffffu;
    const uint32_t b = (uint32_t)w;
    memcpy(&p.value, &b, 4);
    return p;
}

template <typename T>
__device__ __forceinline__ void bk_publish(const BkDesc<T>& d, int64_t tile, uint32_t st, const KPair<T>& p) {
    if constexpr (sizeof(T) == 4) {
        if (d.packed) {
            st_relaxed_u64(d.packed + tile, bk_pack(st, p));
            return;
        }
    }
    uint64_t* w = d.split + tile * BkDesc<T>::WPT;
    const uint64_t hi = (uint64_t)st << 32;
    uint64_t b = 0;
    memcpy(&b, &p.value, sizeof(T));
    st_relaxed_u64(w, hi | p.count);
    st_relaxed_u64(w + 1, hi | (b & 0xFFFFFFFFull));
    if constexpr (sizeof(T) == 8) st_relaxed_u64(w + 2, hi | (b >> 32));
}

// Status of tile p (0 = not ready), and its raw words once ready.
template <typename T>
__device__ __forceinline__ uint32_t bk_poll(const BkDesc<T>& d, int64_t p, BkRaw& r) {
    if constexpr (sizeof(T) == 4) {
        if (d.packed) {
            r.w[0] = ld_relaxed_u64(d.packed + p);
            return (uint32_t)(r.w[0] >> 62);
        }
    }
    const uint64_t* w = d.split + p * BkDesc<T>::WPT;
    r.w[0] = ld_relaxed_u64(w);
    r.w[1] = ld_relaxed_u64(w + 1);
    const uint32_t st = (uint32_t)(r.w[0] >> 32);
    bool same = (uint32_t)(r.w[1] >> 32) == st;
    if constexpr (sizeof(T) == 8) {
        r.w[2] = ld_relaxed_u64(w + 2);
        same = same && (uint32_t)(r.w[2] >> 32) == st;
    }
    return same ? st : 0u;
}
template <typename T>
__device__ __forceinline__ KPair<T> bk_fetch(const BkDesc<T>& d, int64_t, uint32_t, const BkRaw& r) {
    if constexpr (sizeof(T) == 4) {
        if (d.packed) return bk_unpack<T>(r.w[0]);
    }
    KPair<T> v;
    v.count = (uint32_t)r.w[0];
    uint64_t b = r.w[1] & 0xFFFFFFFFull;
    if constexpr (sizeof(T) == 8) b |= r.w[2] << 32;
    memcpy(&v.value, &b, sizeof(T));
    return v;
}

// Warp-wide ordered look-back: the combination of the aggregates of tiles
// [0, tile), same value in every lane.  Lane L inspects tile (window_end - L);
// higher lanes are further left, so the reduction keeps that order.
template <typename Op, typename T>
__device__ KPair<T> bk_lookback(const BkDesc<T>& d, int64_t tile) {
    const int lane = threadIdx.x & 31;
    const uint32_t limit = g_spin_limit;
    KPair<T> acc = kidentity<Op, T>();
    int64_t p = tile - 1 - lane;
    uint32_t spins = 0;
    while (true) {
        BkRaw word{};
        uint32_t st = p >= 0 ? bk_poll(d, p, word) : 2u;
        while (__any_sync(0xffffffffu, st == 0)) {
            if (++spins > limit) {
                if (lane == 0) set_error(LCPP_ERR_LOOKBACK_TIMEOUT);
                return acc;
            }
            if (spins > 64) __nanosleep(spins < 1024 ? 32 : 128);
            if (st == 0) st = bk_poll(d, p, word);
        }
        KPair<T> v = kidentity<Op, T>();
        if (p >= 0) v = bk_fetch(d, p, st, word);
        const uint32_t incl = __ballot_sync(0xffffffffu, st == 2);
        const int first = incl ? __ffs(incl) - 1 : 32;
        if (lane > first) v = kidentity<Op, T>();
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const KPair<T> y = kshfl_down(v, o);
            if (lane + o < 32) v = kcombine<Op, T>(y, v);
        }
        acc = kcombine<Op, T>(kshfl(v, 0), acc);
        if (incl) return acc;
        p -= 32;
    }
}

// Shared-memory layout of a tile array: thread r's ITEMS items occupy CPT
// 16-byte chunks; chunk c of row r is stored at r*CPT + (c ^ swz(r)), which
// spreads the 8 rows a quarter-warp touches over all 32 banks.
template <typename E, int ITEMS>
struct Swz {
    static constexpr int EPC = 16 / sizeof(E);            // elements per chunk
    static constexpr int CPT = ITEMS * sizeof(E) / 16;    // chunks per thread
    static_assert(CPT == 2 || CPT == 4, "2 or 4 chunks per thread");
    static constexpr int ROWS8 = 8 / CPT;                 // rows per 128-byte bank cycle
    __device__ static __forceinline__ int chunk(int r, int c) { return r * CPT + (c ^ ((r / ROWS8) & (CPT - 1))); }
    __device__ static __forceinline__ int elem(int r, int j) { return chunk(r, j / EPC) * EPC + (j % EPC); }
};

// Striped global -> swizzled shared copy of tile items [0, cnt).
template <typename E, int ITEMS>
__device__ __forceinline__ void bk_load(E* s, const E* g, int cnt, bool vec) {
    using S = Swz<E, ITEMS>;
    constexpr int TILE = BK_THREADS * ITEMS;
    if (vec && cnt == TILE) {
        const uint4* gv = reinterpret_cast<const uint4*>(g);
        uint4* sv = reinterpret_cast<uint4*>(s);
        uint4 q[S::CPT];
#pragma unroll
        for (int v = 0; v < S::CPT; ++v) q[v] = ld_stream(gv + v * BK_THREADS + threadIdx.x);
#pragma unroll
        for (int v = 0; v < S::CPT; ++v) {
            const int gi = v * BK_THREADS + threadIdx.x;
            sv[S::chunk(gi / S::CPT, gi % S::CPT)] = q[v];
        }
    } else {
        for (int e = threadIdx.x; e < cnt; e += BK_THREADS) s[S::elem(e / ITEMS, e % ITEMS)] = ldcs(g + e);
    }
}

template <typename E, int ITEMS>
__device__ __forceinline__ void bk_store(E* g, const E* s, int cnt, bool vec) {
    using S = Swz<E, ITEMS>;
    constexpr int TILE = BK_THREADS * ITEMS;
    if (vec && cnt == TILE) {
        uint4* gv = reinterpret_cast<uint4*>(g);
        const uint4* sv = reinterpret_cast<const uint4*>(s);
#pragma unroll
        for (int v = 0; v < S::CPT; ++v) {
            const int gi = v * BK_THREADS + threadIdx.x;
            __stcs(gv + gi, sv[S::chunk(gi / S::CPT, gi % S::CPT)]);
        }
    } else {
        for (int e = threadIdx.x; e < cnt; e += BK_THREADS) stcs(g + e, s[S::elem(e / ITEMS, e % ITEMS)]);
    }
}

// Key equality of the reference's FlagHeads (a != b): bit equality for
// integers, value equality for floats (-0 == +0, NaN never equal).
template <typename K> __device__ __forceinline__ bool key_differs(K a, K b) { return a != b; }

template <typename K, typename T, typename Op, int MODE, int ITEMS>
__global__ void __launch_bounds__(BK_THREADS, 2)
by_key_kernel(const K* __restrict__ keys, const T* values, T* out_values, K* __restrict__ unique_out,
              uint32_t* __restrict__ num_runs_out, uint64_t n, T init, bool vec,
              unsigned int* ticket, BkDesc<T> desc) {
    constexpr int TILE = BK_THREADS * ITEMS;
    using SK = Swz<K, ITEMS>;
    using SV = Swz<T, ITEMS>;
    extern __shared__ __align__(16) unsigned char bk_smem[];
    K* s_keys = reinterpret_cast<K*>(bk_smem);
    T* s_vals = reinterpret_cast<T*>(bk_smem + TILE * sizeof(K));
    __shared__ unsigned int s_tile;
    __shared__ K s_pred;
    __shared__ KPair<T> s_wagg[BK_WARPS];
    __shared__ KPair<T> s_wpre[BK_WARPS];
    __shared__ KPair<T> s_tpre, s_tagg;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, r = threadIdx.x;
    if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1u);
    __syncthreads();
    const int64_t tile = s_tile;
    const uint64_t base = (uint64_t)tile * TILE;
    const int cnt = (int)(n - base < (uint64_t)TILE ? n - base : (uint64_t)TILE);
    if (threadIdx.x == 0 && tile > 0) s_pred = keys[base - 1];
    bk_load<K, ITEMS>(s_keys, keys + base, cnt, vec);
    bk_load<T, ITEMS>(s_vals, values + base, cnt, vec);
    __syncthreads();

    // Blocked items of this thread, head flags, thread aggregate.
    K k[ITEMS];
    T v[ITEMS];
    const int first = r * ITEMS;
#pragma unroll
    for (int c = 0; c < SK::CPT; ++c) {
        const uint4 q = reinterpret_cast<const uint4*>(s_keys)[SK::chunk(r, c)];
        memcpy(&k[c * SK::EPC], &q, 16);
    }
#pragma unroll
    for (int c = 0; c < SV::CPT; ++c) {
        const uint4 q = reinterpret_cast<const uint4*>(s_vals)[SV::chunk(r, c)];
        memcpy(&v[c * SV::EPC], &q, 16);
    }
    if (cnt < TILE) {
#pragma unroll
        for (int j = 0; j < ITEMS; ++j)
            if (first + j >= cnt) v[j] = Op::template identity<T>();
    }
    K kprev0 = r ? s_keys[SK::elem(r - 1, ITEMS - 1)] : s_pred;
    uint32_t flags = 0;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const uint64_t i = base + first + j;
        const K kp = j ? k[j - 1] : kprev0;
        bool head;
        if (MODE == BK_REDUCE) head = i > 0 && i < n && key_differs(k[j], kp);
        else head = i < n && (i == 0 || key_differs(k[j], kp));
        flags |= (uint32_t)head << j;
    }
    KPair<T> agg = kidentity<Op, T>();
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        KPair<T> it;
        it.count = (flags >> j) & 1u;
        it.value = v[j];
        agg = kcombine<Op, T>(agg, it);
    }
    KPair<T> incl = agg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const KPair<T> y = kshfl_up(incl, o);
        if (lane >= o) incl = kcombine<Op, T>(y, incl);
    }
    KPair<T> wex = kshfl_up(incl, 1);
    if (lane == 0) wex = kidentity<Op, T>();
    if (lane == 31) s_wagg[warp] = incl;
    __syncthreads();  // shared key/value staging is free from here on

    if (warp == 0) {
        KPair<T> w = lane < BK_WARPS ? s_wagg[lane] : kidentity<Op, T>();
#pragma unroll
        for (int o = 1; o < BK_WARPS; o <<= 1) {
            const KPair<T> y = kshfl_up(w, o);
            if (lane >= o) w = kcombine<Op, T>(y, w);
        }
        const KPair<T> tagg = kshfl(w, BK_WARPS - 1);
        KPair<T> tpre = kidentity<Op, T>();
        if (tile == 0) {
            if (lane == 0) bk_publish(desc, 0, 2u, tagg);
        } else {
            if (lane == 0) bk_publish(desc, tile, 1u, tagg);
            tpre = bk_lookback<Op, T>(desc, tile);
            if (lane == 0) bk_publish(desc, tile, 2u, kcombine<Op, T>(tpre, tagg));
        }
        KPair<T> wx = kshfl_up(w, 1);
        if (lane == 0) wx = kidentity<Op, T>();
        if (lane < BK_WARPS) s_wpre[lane] = kcombine<Op, T>(tpre, wx);
        if (lane == 0) {
            s_tpre = tpre;
            s_tagg = tagg;
        }
    }
    __syncthreads();

    KPair<T> run = kcombine<Op, T>(s_wpre[warp], wex);
    if (MODE != BK_REDUCE) {
        T o[ITEMS];
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const bool head = (flags >> j) & 1u;
            T oj;
            if (MODE == BK_SCAN_EXCL) {
                oj = head ? init : Op::template apply<T>(run.value, init);
                run.value = head ? v[j] : Op::template apply<T>(run.value, v[j]);
            } else {
                run.value = head ? v[j] : Op::template apply<T>(run.value, v[j]);
                oj = Op::template apply<T>(run.value, init);
            }
            o[j] = oj;
        }
#pragma unroll
        for (int c = 0; c < SV::CPT; ++c) {
            uint4 q;
            memcpy(&q, &o[c * SV::EPC], 16);
            reinterpret_cast<uint4*>(s_vals)[SV::chunk(r, c)] = q;
        }
        __syncthreads();
        bk_store<T, ITEMS>(out_values + base, s_vals, cnt, vec);
    } else {
        const uint32_t c0 = s_tpre.count;
        const uint32_t ntile = s_tagg.count;
        T* s_agg = s_vals;       // compacted runs of this tile, dense from 0
        K* s_uk = s_keys;
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const bool head = (flags >> j) & 1u;
            if (head) {
                const uint32_t pos = run.count - c0;
                s_uk[pos] = j ? k[j - 1] : kprev0;
                s_agg[pos] = run.value;
            }
            run.count += head;
            run.value = head ? v[j] : Op::template apply<T>(run.value, v[j]);
            if (base + first + j == n - 1) {  // the run that ends the input
                unique_out[run.count] = k[j];
                out_values[run.count] = run.value;
                *num_runs_out = run.count + 1;
            }
        }
        __syncthreads();
        for (uint32_t e = threadIdx.x; e < ntile; e += BK_THREADS) {
            unique_out[c0 + e] = s_uk[e];
            out_values[c0 + e] = s_agg[e];
        }
    }
}

// ---------------------------------------------------------------------------
// Pipelined persistent form (16-byte-aligned keys, values and outputs).
//
// Persistent CTAs (2 per SM, 512 threads) stream tiles through three
// shared-memory stages filled by TMA bulk copies (cp.async.bulk, this GPU's
// memory only, no multicast).  A stage holds the tile's keys, its values and
// the 16 bytes of keys just before the tile (the predecessor key), all landed
// on one mbarrier.  As in the pipelined plain scan, a CTA publishes the
// aggregate of its NEXT tile as soon as that tile lands, before it resolves
// the look-back of its current tile, so partial descriptors run one tile
// ahead of the scan frontier.  Per-thread state of a tile (head-flag mask and
// the thread's exclusive pair within its warp) stays in registers between the
// two phases; per-warp prefixes of each stage stay in shared memory.
// Each thread owns 32 bytes of the wider of key and value: 8 items for
// 4-byte keys and values, 4 items otherwise (tiles of 4096 / 2048 items).
// ---------------------------------------------------------------------------
constexpr int BKP_STAGES = 3;
constexpr int BKP_CTAS_PER_SM = 2;
constexpr int BK_DESC_TILE = 2048;  // smallest tile of any by-key kernel: sizes the descriptors

template <typename K, typename T>
struct BkpShape {
    static constexpr int W = sizeof(K) > sizeof(T) ? sizeof(K) : sizeof(T);
    static constexpr int ITEMS = 32 / W;
    static constexpr int TILE = BK_THREADS * ITEMS;
    static constexpr int KBYTES = TILE * sizeof(K);
    static constexpr int VBYTES = TILE * sizeof(T);
    static constexpr int STAGE = KBYTES + VBYTES + 16;  // + predecessor keys
    static constexpr int KCH = ITEMS * sizeof(K) / 16;  // 16-byte chunks per thread
    static constexpr int VCH = ITEMS * sizeof(T) / 16;
    static_assert(TILE >= BK_DESC_TILE, "descriptor array sized for BK_DESC_TILE");
};

template <typename K, typename T, typename Op, int MODE>
__global__ void __launch_bounds__(BK_THREADS, BKP_CTAS_PER_SM)
by_key_pipe_kernel(const K* keys, const T* values, T* out_values, K* __restrict__ unique_out,
                   uint32_t* __restrict__ num_runs_out, uint64_t n, uint64_t num_tiles, T init,
                   unsigned int* ticket, BkDesc<T> desc) {
    using S = BkpShape<K, T>;
    constexpr int ITEMS = S::ITEMS, TILE = S::TILE;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t s_bar[BKP_STAGES];
    __shared__ unsigned int s_tile[BKP_STAGES];
    __shared__ KPair<T> s_wagg[BKP_STAGES][BK_WARPS];  // indexed by stage: no barrier guards their reuse
    __shared__ KPair<T> s_wpre[BKP_STAGES][BK_WARPS];
    __shared__ KPair<T> s_tagg[BKP_STAGES];
    __shared__ KPair<T> s_tpre[BKP_STAGES];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t full_tiles = n / TILE;
    const uint32_t limit = g_spin_limit;
    uint32_t phase[BKP_STAGES] = {};

    auto stage_keys = [&](int st) { return reinterpret_cast<K*>(smem + st * S::STAGE); };
    auto stage_vals = [&](int st) { return reinterpret_cast<T*>(smem + st * S::STAGE + S::KBYTES); };
    auto stage_pred = [&](int st) { return reinterpret_cast<K*>(smem + st * S::STAGE + S::KBYTES + S::VBYTES); };

    auto issue = [&](unsigned int t, int st) {  // thread 0
        if (t < full_tiles) {
            fence_proxy_async_smem();
            const uint64_t base = (uint64_t)t * TILE;
            mbar_arrive_expect_tx(&s_bar[st], S::KBYTES + S::VBYTES + (t ? 16 : 0));
            bulk_load(stage_keys(st), keys + base, S::KBYTES, &s_bar[st]);
            bulk_load(stage_vals(st), values + base, S::VBYTES, &s_bar[st]);
            if (t) bulk_load(stage_pred(st), reinterpret_cast<const char*>(keys + base) - 16, 16, &s_bar[st]);
        }
    };

    // Blocked items of thread tid in stage st.
    auto read_items = [&](int st, K (&k)[ITEMS], T (&v)[ITEMS]) {
#pragma unroll
        for (int c = 0; c < S::KCH; ++c) {
            const uint4 q = reinterpret_cast<const uint4*>(stage_keys(st))[tid * S::KCH + c];
            memcpy(&k[c * (16 / sizeof(K))], &q, 16);
        }
#pragma unroll
        for (int c = 0; c < S::VCH; ++c) {
            const uint4 q = reinterpret_cast<const uint4*>(stage_vals(st))[tid * S::VCH + c];
            memcpy(&v[c * (16 / sizeof(T))], &q, 16);
        }
    };
    auto prev_key = [&](int st) -> K {
        return tid ? stage_keys(st)[tid * ITEMS - 1] : stage_pred(st)[16 / sizeof(K) - 1];
    };

    // Phase 1 of tile t in stage st: wait for its data, head flags, pair
    // scans, publish the tile aggregate.  Returns the thread's flag mask and
    // its exclusive pair within the warp.
    auto aggregate = [&](uint64_t t, int st, uint32_t& flags, KPair<T>& wex) {
        const uint64_t base = t * TILE;
        if (t < full_tiles) {
            if (!mbar_wait(&s_bar[st], phase[st], limit)) set_error(LCPP_ERR_LOOKBACK_TIMEOUT);
            phase[st] ^= 1;
        } else {  // ragged last tile: guarded copy
            K* sk = stage_keys(st);
            T* sv = stage_vals(st);
            for (int i = tid; i < TILE; i += BK_THREADS) {
                const uint64_t g = base + i;
                if (g < n) {
                    sk[i] = keys[g];
                    sv[i] = values[g];
                }
            }
            if (tid == 0 && t > 0) stage_pred(st)[16 / sizeof(K) - 1] = keys[base - 1];
            __syncthreads();
        }
        K k[ITEMS];
        T v[ITEMS];
        read_items(st, k, v);
        const K kp0 = prev_key(st);
        flags = 0;
        KPair<T> agg = kidentity<Op, T>();
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const uint64_t i = base + (uint64_t)tid * ITEMS + j;
            const K kp = j ? k[j - 1] : kp0;
            bool head;
            if (MODE == BK_REDUCE) head = i > 0 && i < n && key_differs(k[j], kp);
            else head = i < n && (i == 0 || key_differs(k[j], kp));
            flags |= (uint32_t)head << j;
            KPair<T> it;
            it.count = head;
            it.value = i < n ? v[j] : Op::template identity<T>();
            agg = kcombine<Op, T>(agg, it);
        }
        KPair<T> incl = agg;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const KPair<T> y = kshfl_up(incl, o);
            if (lane >= o) incl = kcombine<Op, T>(y, incl);
        }
        wex = kshfl_up(incl, 1);
        if (lane == 0) wex = kidentity<Op, T>();
        if (lane == 31) s_wagg[st][warp] = incl;
        __syncthreads();
        if (warp == 0) {
            KPair<T> w = lane < BK_WARPS ? s_wagg[st][lane] : kidentity<Op, T>();
#pragma unroll
            for (int o = 1; o < BK_WARPS; o <<= 1) {
                const KPair<T> y = kshfl_up(w, o);
                if (lane >= o) w = kcombine<Op, T>(y, w);
            }
            KPair<T> wx = kshfl_up(w, 1);
            if (lane == 0) wx = kidentity<Op, T>();
            if (lane < BK_WARPS) s_wpre[st][lane] = wx;
            if (lane == BK_WARPS - 1) {
                s_tagg[st] = w;
                bk_publish(desc, (int64_t)t, t == 0 ? 2u : 1u, w);
            }
        }
    };

    // Phase 2 of tile t: look-back, outputs.
    auto scan_tile = [&](uint64_t t, int st, uint32_t flags, const KPair<T>& wex) {
        const uint64_t base = t * TILE;
        const bool full = t < full_tiles;
        // s_wpre / s_tagg of this stage were written one iteration earlier
        if (warp == 0) {
            KPair<T> tpre = kidentity<Op, T>();
            if (t != 0) {
                tpre = bk_lookback<Op, T>(desc, (int64_t)t);
                if (lane == 0) bk_publish(desc, (int64_t)t, 2u, kcombine<Op, T>(tpre, s_tagg[st]));
            }
            if (lane == 0) s_tpre[st] = tpre;
        }
        __syncthreads();
        const KPair<T> tpre = s_tpre[st];
        KPair<T> run = kcombine<Op, T>(kcombine<Op, T>(tpre, s_wpre[st][warp]), wex);
        K k[ITEMS];
        T v[ITEMS];
        read_items(st, k, v);
        if (MODE != BK_REDUCE) {
            T o[ITEMS];
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) {
                const bool head = (flags >> j) & 1u;
                if (MODE == BK_SCAN_EXCL) {
                    o[j] = head ? init : Op::template apply<T>(run.value, init);
                    run.value = head ? v[j] : Op::template apply<T>(run.value, v[j]);
                } else {
                    run.value = head ? v[j] : Op::template apply<T>(run.value, v[j]);
                    o[j] = Op::template apply<T>(run.value, init);
                }
            }
            if (full) {
#pragma unroll
                for (int c = 0; c < S::VCH; ++c) {
                    uint4 q;
                    memcpy(&q, &o[c * (16 / sizeof(T))], 16);
                    reinterpret_cast<uint4*>(stage_vals(st))[tid * S::VCH + c] = q;
                }
                fence_proxy_async_smem();
                __syncthreads();
                if (tid == 0) {
                    bulk_store(out_values + base, stage_vals(st), S::VBYTES);
                    bulk_commit();
                }
            } else {
#pragma unroll
                for (int j = 0; j < ITEMS; ++j) {
                    const uint64_t i = base + (uint64_t)tid * ITEMS + j;
                    if (i < n) out_values[i] = o[j];
                }
            }
        } else {
            const K kp0 = prev_key(st);
            const uint32_t c0 = tpre.count;
            const uint32_t ntile = s_tagg[st].count;
            __syncthreads();  // every thread holds its items: the stage is free for compaction
            K* s_uk = stage_keys(st);
            T* s_agg = stage_vals(st);
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) {
                const bool head = (flags >> j) & 1u;
                if (head) {
                    const uint32_t pos = run.count - c0;
                    s_uk[pos] = j ? k[j - 1] : kp0;
                    s_agg[pos] = run.value;
                }
                run.count += head;
                run.value = head ? v[j] : Op::template apply<T>(run.value, v[j]);
                if (base + (uint64_t)tid * ITEMS + j == n - 1) {  // the run that ends the input
                    unique_out[run.count] = k[j];
                    out_values[run.count] = run.value;
                    *num_runs_out = run.count + 1;
                }
            }
            __syncthreads();
            for (uint32_t e = tid; e < ntile; e += BK_THREADS) {
                unique_out[c0 + e] = s_uk[e];
                out_values[c0 + e] = s_agg[e];
            }
        }
    };

    if (tid == 0) {
        for (int i = 0; i < BKP_STAGES; ++i) mbar_init(&s_bar[i], 1);
        fence_mbar_init();
        for (int i = 0; i < BKP_STAGES; ++i) {
            const unsigned int t = atomicAdd(ticket, 1u);
            s_tile[i] = t;
            issue(t, i);
        }
    }
    __syncthreads();

    uint64_t c = s_tile[0];
    int st = 0;
    uint32_t fl_c = 0, fl_n = 0;
    KPair<T> wx_c = kidentity<Op, T>(), wx_n = kidentity<Op, T>();
    if (c < num_tiles) aggregate(c, 0, fl_c, wx_c);
    while (c < num_tiles) {
        const int nst = st + 1 == BKP_STAGES ? 0 : st + 1;
        const uint64_t nt = s_tile[nst];
        // The ticket for the stage this iteration frees is taken now, so the
        // atomic's round trip overlaps the two phases below.  The stage's new
        // ticket is read two iterations later, past this iteration's barriers.
        const unsigned int pref = tid == 0 ? atomicAdd(ticket, 1u) : 0u;
        if (nt < num_tiles) aggregate(nt, nst, fl_n, wx_n);
        scan_tile(c, st, fl_c, wx_c);
        if (MODE == BK_REDUCE) __syncthreads();  // the compacted runs have left the stage
        if (tid == 0) {
            s_tile[st] = pref;
            bulk_wait_read_all();  // this stage's bulk store has read it
            issue(pref, st);
        }
        c = nt;
        st = nst;
        fl_c = fl_n;
        wx_c = wx_n;
    }
    if (tid == 0) bulk_wait_all();
}

template <typename K, typename T>
constexpr int bk_items() { return (sizeof(K) == 4 && sizeof(T) == 4) ? 16 : 8; }

template <typename K, typename T, typename Op, int MODE>
static lcpp_status bk_launch(const void* keys, const void* values, void* out_values, void* unique_out,
                             uint32_t* num_runs, uint64_t n, T init, void* temp, cudaStream_t s) {
    constexpr int ITEMS = bk_items<K, T>();
    constexpr int TILE = BK_THREADS * ITEMS;
    const uint64_t tiles = ceil_div(n, BK_DESC_TILE);  // descriptor slots (>= tiles of either kernel)
    unsigned int* ticket = (unsigned int*)temp;
    BkDesc<T> d;
    const bool packed = sizeof(T) == 4 && n < (1ull << 30);
    uint64_t* words = (uint64_t*)((char*)temp + BK_HDR);
    d.packed = packed ? words : nullptr;
    d.split = packed ? nullptr : words;
    if (cudaMemsetAsync(temp, 0, BK_HDR + tiles * 8 * (packed ? 1 : BkDesc<T>::WPT), s) != cudaSuccess)
        return LCPP_ERR_CUDA;
    const bool vec = ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(values) |
                       (MODE == BK_REDUCE ? 0 : reinterpret_cast<uintptr_t>(out_values))) & 15) == 0;
    ProfScope ps(MODE == BK_REDUCE ? "reduce_by_key" : "scan_by_key", s);
    if (vec) {
        using SP = BkpShape<K, T>;
        const uint64_t ptiles = ceil_div(n, SP::TILE);
        const size_t psmem = (size_t)BKP_STAGES * SP::STAGE;
        uint64_t grid = (uint64_t)device_info().sms * BKP_CTAS_PER_SM;
        if (grid > ceil_div(ptiles, 2)) grid = ceil_div(ptiles, 2);
        auto pk = by_key_pipe_kernel<K, T, Op, MODE>;
        if (cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem) != cudaSuccess)
            return LCPP_ERR_CUDA;
        pk<<<(unsigned)grid, BK_THREADS, psmem, s>>>((const K*)keys, (const T*)values, (T*)out_values,
                                                      (K*)unique_out, num_runs, n, ptiles, init, ticket, d);
        count_launch();
        return check_launch();
    }
    const size_t smem = (size_t)TILE * (sizeof(K) + sizeof(T));
    auto kern = by_key_kernel<K, T, Op, MODE, ITEMS>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return LCPP_ERR_CUDA;
    kern<<<(unsigned)ceil_div(n, TILE), BK_THREADS, smem, s>>>((const K*)keys, (const T*)values, (T*)out_values,
                                                   (K*)unique_out, num_runs, n, init, vec, ticket, d);
    count_launch();
    return check_launch();
}

static size_t bk_temp_bytes(int key_dtype, int value_dtype, uint64_t n) {
    const size_t ks = lcpp_dtype_size(key_dtype), vs = lcpp_dtype_size(value_dtype);
    if (!ks || !vs) return 0;
    const uint64_t tiles = ceil_div(n ? n : 1, BK_DESC_TILE);
    return BK_HDR + align_up(tiles * 8 * (vs == 8 ? 3 : 2), 256);  // packed form: 1 word per tile
}

// Key dispatch: integer keys compare by bits, float keys by value.
template <typename F>
static lcpp_status dispatch_key(int key_dtype, F&& f) {
    switch (key_dtype) {
        case LCPP_I32: case LCPP_U32: return f((uint32_t)0);
        case LCPP_I64: case LCPP_U64: return f((uint64_t)0);
        case LCPP_F32: return f((float)0);
        case LCPP_F64: return f((double)0);
        default: return LCPP_ERR_INVALID_ARG;
    }
}

template <int MODE>
static lcpp_status bk_dispatch(int op, int key_dtype, int value_dtype, const void* keys, const void* values,
                               void* out_values, void* unique_out, uint32_t* num_runs, uint64_t n,
                               const void* init, void* temp, cudaStream_t s) {
    return dispatch_key(key_dtype, [&](auto kz) -> lcpp_status {
        using K = decltype(kz);
        return dispatch_dtype(value_dtype, [&](auto vz) -> lcpp_status {
            using T = decltype(vz);
            auto go = [&](auto opv) -> lcpp_status {
                using Op = decltype(opv);
                const T iv = init ? *(const T*)init : Op::template identity<T>();
                return bk_launch<K, T, Op, MODE>(keys, values, out_values, unique_out, num_runs, n, iv, temp, s);
            };
            switch (op) {
                case LCPP_OP_SUM: return go(OpSum{});
                case LCPP_OP_MIN: return go(OpMin{});
                default: return go(OpMax{});
            }
        });
    });
}

}  // namespace lcpp

using namespace lcpp;

extern "C" size_t lcpp_scan_by_key_temp_bytes(int key_dtype, int value_dtype, uint64_t n) {
    return bk_temp_bytes(key_dtype, value_dtype, n);
}

extern "C" lcpp_status lcpp_scan_by_key(int kind, int op, int key_dtype, int value_dtype, const void* keys,
                                        const void* values_in, void* values_out, uint64_t n,
                                        const void* init, void* temp, size_t temp_bytes, void* stream) {
    if ((kind != LCPP_SCAN_EXCLUSIVE && kind != LCPP_SCAN_INCLUSIVE) || op < 0 || op > 2) return LCPP_ERR_INVALID_ARG;
    const size_t need = bk_temp_bytes(key_dtype, value_dtype, n);
    if (!need || n > 0xffffffffull) return LCPP_ERR_INVALID_ARG;
    if (n == 0) return LCPP_OK;
    if (!keys || !values_in || !values_out) return LCPP_ERR_INVALID_ARG;
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    cudaStream_t s = (cudaStream_t)stream;
    if (kind == LCPP_SCAN_INCLUSIVE)
        return bk_dispatch<BK_SCAN_INCL>(op, key_dtype, value_dtype, keys, values_in, values_out, nullptr, nullptr,
                                         n, init, temp, s);
    return bk_dispatch<BK_SCAN_EXCL>(op, key_dtype, value_dtype, keys, values_in, values_out, nullptr, nullptr, n,
                                     init, temp, s);
}

extern "C" size_t lcpp_reduce_by_key_temp_bytes(int key_dtype, int value_dtype, uint64_t n) {
    return bk_temp_bytes(key_dtype, value_dtype, n);
}

extern "C" lcpp_status lcpp_reduce_by_key(int op, int key_dtype, int value_dtype, const void* keys_in,
                                          const void* values_in, void* unique_out, void* aggregates_out,
                                          uint32_t* num_runs_out, uint64_t n, void* temp, size_t temp_bytes,
                                          void* stream) {
    if (op < 0 || op > 2) return LCPP_ERR_INVALID_ARG;
    const size_t need = bk_temp_bytes(key_dtype, value_dtype, n);
    if (!need || n > 0xffffffffull || !num_runs_out) return LCPP_ERR_INVALID_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0)
        return cudaMemsetAsync(num_runs_out, 0, sizeof(uint32_t), s) == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
    if (!keys_in || !values_in || !unique_out || !aggregates_out) return LCPP_ERR_INVALID_ARG;
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    return bk_dispatch<BK_REDUCE>(op, key_dtype, value_dtype, keys_in, values_in, aggregates_out, unique_out,
                                  num_runs_out, n, nullptr, temp, s);
}
