// DeviceRadixSort for sm_100a: onesweep LSD radix sort (Adinets & Merrill
// 2022), the algorithm of the reference's onesweep_radix_sort
// (src/lcpp/device/device_radix_sort.h:187-378) with its histogram agent
// (src/lcpp/agent/agent_radix_sort_histogram.h:45-198), bins exclusive sum
// (src/lcpp/device/details/radix_sort.h:82-123), onesweep pass agent
// (src/lcpp/agent/agent_radix_sort_onesweep.h:43-500) and match-based block
// rank (src/lcpp/block/block_radix_rank.h:66-336).  Key bit ordering follows
// Traits::TwiddleIn (src/lcpp/common/util_type.h:89-176) and
// ProcessFloatMinusZero (src/lcpp/agent/radix_rank_sort_operations.h:30-43).
//
// B200 design:
//  * One upfront histogram kernel reads every key once and counts the digits
//    of all passes into lane-private shared-memory counter columns (no bank
//    conflicts, skewed keys included), then one tiny kernel turns the counts
//    into per-pass digit starts.
//  * One onesweep kernel per 8-bit pass: 512 threads x 16 keys (8 for 64-bit
//    keys) per tile, tile ids from an atomic ticket, warp-striped coalesced
//    loads, values of full tiles prefetched into shared memory by cp.async,
//    per-warp digit counts published to the look-back before ranking, the
//    per-digit windowed look-back (one 32-bit word per (tile, digit)
//    {flags:2 | count:30}, 64-bit words when n >= 2^30) overlapped with the
//    ranking of the other warps, stable ranking through per-warp atomicOr
//    lane masks per digit, then keys and values placed in shared memory in
//    digit order and written out with consecutive threads on consecutive
//    addresses.
//  * All look-back buffers of a sort are zeroed by one memset; no per-pass
//    reset kernels (the reference resets 1 KiB per tile every pass).
//  * Sizes are 64-bit in the ABI; no 2^28 "portions" (the reference's portion
//    hand-off at agent_radix_sort_onesweep.h:322 is not reproduced).
//  * Bounded look-back waits: after g_spin_limit polls a tile latches
//    LCPP_ERR_LOOKBACK_TIMEOUT and proceeds (no trap, no hang).
#include "common.cuh"
#include <type_traits>

namespace lcpp {

constexpr int RS_BITS = 8;
constexpr int RS_DIGITS = 1 << RS_BITS;
#ifndef LCPP_RS_THREADS_CT
#define LCPP_RS_THREADS_CT 512
#endif
constexpr int RS_THREADS = LCPP_RS_THREADS_CT;
constexpr int RS_WARPS = RS_THREADS / 32;
constexpr int RS_MAX_PASSES = 8;
constexpr int RS_LB_WINDOW = 8;  // predecessor words loaded per look-back step

struct NoValue {};

// Keys per thread of a onesweep tile, by the bytes an item moves (key +
// value): a tile stages 64-72 KiB of keys and values, so two CTAs fit an SM
// beside the rank words, and fewer, larger tiles shorten the look-back
// chains (keys-only u32: 32; u32 pairs or u64 keys only: 18; one 8-byte and
// one 4-byte half: 12; 16-byte pairs: 8).  LCPP_RS_I8 overrides the 8-byte case.
#ifndef LCPP_RS_I8
#define LCPP_RS_I8 18
#endif
// Passes over precomputed digits (DIG) also stage one digit byte per item, so
// their tiles are smaller where the 8-byte and 4-byte sizes would not fit two
// CTAs per SM.
constexpr int rs_items_for(size_t key_bytes, size_t value_bytes, bool dig = false) {
    return key_bytes + value_bytes <= 4 ? (dig ? 28 : 32)
         : key_bytes + value_bytes <= 8 ? (dig ? 16 : LCPP_RS_I8)
         : key_bytes + value_bytes <= 12 ? 12 : 8;
}
template <typename KB, typename VB, bool DIG = false> struct RsItems {
    static constexpr int value = rs_items_for(sizeof(KB), std::is_same<VB, NoValue>::value ? 0 : sizeof(VB), DIG);
};

// Map key bits to an unsigned order-preserving image (ascending), or its
// complement for descending.  KIND: 0 unsigned, 1 signed, 2 floating point.
template <typename KB, int KIND, bool DESC>
__device__ __forceinline__ KB ordered_bits(KB k) {
    constexpr KB HIGH = KB(1) << (sizeof(KB) * 8 - 1);
    KB o;
    if (KIND == 0) {
        o = k;
    } else if (KIND == 1) {
        o = k ^ HIGH;
    } else {
        o = (k & HIGH) ? KB(~k) : KB(k ^ HIGH);
        if (o == KB(~HIGH)) o = HIGH;  // -0.0 sorts as +0.0
    }
    return DESC ? KB(~o) : o;
}

template <typename KB, int KIND, bool DESC>
__device__ __forceinline__ uint32_t digit_of(KB k, uint32_t shift, uint32_t mask) {
    return (uint32_t)(ordered_bits<KB, KIND, DESC>(k) >> shift) & mask;
}

// Histogram of all passes' digits with lane-private counter columns: counter
// (pass, digit) has COLS copies and lane L adds into copy L % COLS, so the
// 32 atomics of a warp instruction fall into distinct banks whatever the
// digits (skewed inputs included) — the shared-atomic bank conflicts that
// bound a single-copy histogram disappear.  One 1024-thread CTA per SM,
// 128 KiB of counters.  bins[p*256 + d] += count.
constexpr int HISTC_THREADS = 1024;
template <typename KB> struct HistCols { static constexpr int value = sizeof(KB) == 4 ? 32 : 16; };
template <typename KB>
constexpr size_t histc_smem_bytes() {
    return (size_t)(sizeof(KB) * 8 / RS_BITS) * RS_DIGITS * HistCols<KB>::value * 4;
}

template <typename KB, int KIND, bool DESC>
__global__ void __launch_bounds__(HISTC_THREADS, 1)
rs_histogram_cols_kernel(const KB* __restrict__ keys, uint64_t n, uint32_t* __restrict__ bins,
                         uint32_t begin_bit, uint32_t end_bit, uint32_t passes) {
    constexpr int COLS = HistCols<KB>::value;
    extern __shared__ __align__(16) uint32_t hc[];  // [passes][256][COLS]
    const uint32_t words = passes * RS_DIGITS * COLS;
    for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) hc[i] = 0;
    __syncthreads();
    const uint32_t col = threadIdx.x & (COLS - 1);

    auto count = [&](KB k) {
        const KB o = ordered_bits<KB, KIND, DESC>(k);
#pragma unroll
        for (uint32_t p = 0; p < RS_MAX_PASSES; ++p) {
            if (p >= passes) break;
            const uint32_t shift = begin_bit + p * RS_BITS;
            const uint32_t mask = (1u << min((uint32_t)RS_BITS, end_bit - shift)) - 1u;
            const uint32_t d = (uint32_t)(o >> shift) & mask;
            atomicAdd(&hc[(p * RS_DIGITS + d) * COLS + col], 1u);
        }
    };

    constexpr int VEC = 16 / sizeof(KB);
    constexpr int HU = 4;
    const bool aligned = (reinterpret_cast<uintptr_t>(keys) & 15) == 0;
    const uint64_t nvec = aligned ? n / VEC : 0;
    const uint4* vk = reinterpret_cast<const uint4*>(keys);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + (HU - 1) * stride < nvec; i += HU * stride) {
        uint4 q[HU];
#pragma unroll
        for (int u = 0; u < HU; ++u) q[u] = ld_stream(vk + i + u * stride);
#pragma unroll
        for (int u = 0; u < HU; ++u) {
            const KB* e = reinterpret_cast<const KB*>(&q[u]);
#pragma unroll
            for (int v = 0; v < VEC; ++v) count(e[v]);
        }
    }
    for (; i < nvec; i += stride) {
        const uint4 q = ld_stream(vk + i);
        const KB* e = reinterpret_cast<const KB*>(&q);
#pragma unroll
        for (int v = 0; v < VEC; ++v) count(e[v]);
    }
    for (uint64_t t = nvec * VEC + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride)
        count(keys[t]);
    __syncthreads();
    // Fold the columns; thread j starts at column j % COLS so reads spread over the banks.
    for (uint32_t b = threadIdx.x; b < passes * RS_DIGITS; b += blockDim.x) {
        uint32_t sum = 0;
#pragma unroll
        for (int c = 0; c < COLS; ++c) sum += hc[b * COLS + ((c + b) & (COLS - 1))];
        if (sum) atomicAdd(bins + b, sum);
    }
}

// In-place exclusive scan of each pass's 256 counts (one CTA per pass), and
// identity[p] = 1 when one digit of pass p holds all n items (the pass is
// then the identity permutation).
__global__ void __launch_bounds__(RS_DIGITS) rs_bins_scan_kernel(uint32_t* bins, uint64_t n, uint32_t* identity) {
    __shared__ uint32_t s_w[RS_DIGITS / 32];
    uint32_t* b = bins + blockIdx.x * RS_DIGITS;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t c = b[threadIdx.x];
    const int one_digit = __syncthreads_or((uint64_t)c == n);
    if (threadIdx.x == 0) identity[blockIdx.x] = one_digit ? 1u : 0u;
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_w[warp] = incl;
    __syncthreads();
    uint32_t wpre = 0;
    for (int w = 0; w < warp; ++w) wpre += s_w[w];
    b[threadIdx.x] = wpre + incl - c;
}

// Counts of precomputed one-byte digits (the DIG passes): lane-private
// columns as above, 16 digits per 128-bit load.  bins[d] += count.
__global__ void __launch_bounds__(HISTC_THREADS, 1)
rs_digit_hist_kernel(const uint8_t* __restrict__ digits, uint64_t n, uint32_t* __restrict__ bins) {
    __shared__ uint32_t hc[RS_DIGITS * 32];
    for (uint32_t i = threadIdx.x; i < RS_DIGITS * 32; i += blockDim.x) hc[i] = 0;
    __syncthreads();
    const uint32_t col = threadIdx.x & 31;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t gtid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool aligned = (reinterpret_cast<uintptr_t>(digits) & 15) == 0;
    const uint64_t nvec = aligned ? n / 16 : 0;
    for (uint64_t i = gtid; i < nvec; i += stride) {
        const uint4 q = ld_stream(reinterpret_cast<const uint4*>(digits) + i);
        const uint8_t* e = reinterpret_cast<const uint8_t*>(&q);
#pragma unroll
        for (int v = 0; v < 16; ++v) atomicAdd(&hc[e[v] * 32 + col], 1u);
    }
    for (uint64_t t = nvec * 16 + gtid; t < n; t += stride) atomicAdd(&hc[digits[t] * 32 + col], 1u);
    __syncthreads();
    for (uint32_t b = threadIdx.x; b < RS_DIGITS; b += blockDim.x) {
        uint32_t sum = 0;
#pragma unroll
        for (int c = 0; c < 32; ++c) sum += hc[b * 32 + ((c + b) & 31)];
        if (sum) atomicAdd(bins + b, sum);
    }
}

// ---------------------------------------------------------------------------
// Look-back words: {INCLUSIVE | PARTIAL | count} in 32 or 64 bits.
// ---------------------------------------------------------------------------
template <typename W> struct LbFlags;
template <> struct LbFlags<uint32_t> {
    static constexpr uint32_t PART = 1u << 30, INCL = 1u << 31, MASK = PART - 1;
};
template <> struct LbFlags<uint64_t> {
    static constexpr uint64_t PART = 1ull << 62, INCL = 1ull << 63, MASK = PART - 1;
};
__device__ __forceinline__ uint32_t lb_load(const uint32_t* p) { return ld_relaxed_u32(p); }
__device__ __forceinline__ uint64_t lb_load(const uint64_t* p) { return ld_relaxed_u64(p); }
__device__ __forceinline__ void lb_store(uint32_t* p, uint32_t v) { st_relaxed_u32(p, v); }
__device__ __forceinline__ void lb_store(uint64_t* p, uint64_t v) { st_relaxed_u64(p, v); }

struct RsPass {
    const void* keys_in;
    void* keys_out;
    const void* vals_in;
    void* vals_out;
    uint64_t n;
    uint32_t shift;
    uint32_t mask;
    const uint32_t* bins;   // 256 global digit starts of this pass
    void* lookback;         // tiles x 256 words, zeroed
    uint32_t* ticket;       // zeroed
    const uint32_t* identity;  // nonzero: this pass is the identity permutation
    const uint8_t* digits;      // DIG kernels: precomputed digit of every item (no key bits used)
};

template <typename KB, typename VB, int THREADS, bool DIG = false>
constexpr size_t rs_smem_bytes() {
    constexpr int TILE = THREADS * RsItems<KB, VB, DIG>::value;
    return (DIG ? (size_t)TILE : 0) + (size_t)TILE * sizeof(KB) +
           (std::is_same<VB, NoValue>::value ? 0 : (size_t)TILE * sizeof(VB)) +
           (size_t)(THREADS / 32) * RS_DIGITS * 4 * 2 + RS_DIGITS * 4 * 2 + 64;
}


// Coalesced copy of items [base, base + count) (16-byte vectors when aligned).
template <typename E>
__device__ __forceinline__ void rs_copy_tile(const void* src, void* dst, uint64_t base, uint32_t count, int tid,
                                             int threads) {
    const E* s = reinterpret_cast<const E*>(src) + base;
    E* d = reinterpret_cast<E*>(dst) + base;
    constexpr uint32_t V = 16 / sizeof(E);
    const bool vec = ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) == 0;
    uint32_t done = 0;
    if (vec) {
        const uint32_t nv = count / V;
        for (uint32_t i = tid; i < nv; i += threads)
            __stcs(reinterpret_cast<uint4*>(d) + i, ld_stream(reinterpret_cast<const uint4*>(s) + i));
        done = nv * V;
    }
    for (uint32_t i = done + tid; i < count; i += threads) stcs(d + i, ldcs(s + i));
}

template <typename KB, typename VB, typename W, int KIND, bool DESC, int THREADS, bool DIG = false>
__global__ void __launch_bounds__(THREADS, 1024 / THREADS) rs_onesweep_kernel(RsPass a) {
    constexpr int RS_WARPS = THREADS / 32;
    constexpr int ITEMS = RsItems<KB, VB, DIG>::value;
    constexpr int TILE = THREADS * ITEMS;
    constexpr bool HAS_V = !std::is_same<VB, NoValue>::value;
    using F = LbFlags<W>;

    extern __shared__ __align__(16) unsigned char smem[];
    KB* s_keys = reinterpret_cast<KB*>(smem);
    unsigned char* p = smem + (size_t)TILE * sizeof(KB);
    VB* s_vals = reinterpret_cast<VB*>(p);
    if constexpr (HAS_V) p += (size_t)TILE * sizeof(VB);
    // One word per (half-warp, digit): {lane mask of the half-warp : 16 | counter : 16}.
    constexpr int RS_HALVES = 2 * RS_WARPS;
    uint32_t* s_wc = reinterpret_cast<uint32_t*>(p);          // [RS_HALVES][256]
    uint32_t* s_gbase = s_wc + RS_HALVES * RS_DIGITS;        // [256]
    uint32_t* s_misc = s_gbase + RS_DIGITS;                  // [0] tile id, [1..8] warp sums
    uint8_t* s_dig = reinterpret_cast<uint8_t*>(s_misc + 16);  // DIG: digit per tile slot

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_misc[0] = atomicAdd(a.ticket, 1u);
    for (int i = tid; i < RS_HALVES * RS_DIGITS; i += THREADS) s_wc[i] = 0;
    // A pass in which one digit holds every item (skewed keys: e.g. the high
    // digits of keys with 8 bits of entropy) is the identity permutation.  The
    // flag is loaded now and looked at once the keys are in registers.
    const uint32_t identity_pass = *a.identity;
    __syncthreads();
    const uint64_t tile = s_misc[0];
    const uint64_t tile_base = tile * TILE;
    const uint64_t rem = a.n - tile_base;
    const uint32_t num_valid = rem < (uint64_t)TILE ? (uint32_t)rem : (uint32_t)TILE;

    const KB* kin = reinterpret_cast<const KB*>(a.keys_in);
    // Each half-warp owns ITEMS * 16 consecutive items of the tile (item i of
    // lane hl at hbase + i * 16 + hl) and ranks them with its own counters.
    const uint32_t half = (uint32_t)lane >> 4, hl = (uint32_t)lane & 15;
    const uint32_t hbase = (uint32_t)warp * (ITEMS * 32) + half * (ITEMS * 16) + hl;

    // ---- load (warp-striped) -------------------------------------------------
    KB key[ITEMS];
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const uint32_t li = hbase + i * 16;
        key[i] = li < num_valid ? ldcs(kin + tile_base + li) : KB(0);
    }
    if (identity_pass) {  // keys back out where they came from, values copied; no rank, no look-back
        KB* kout0 = reinterpret_cast<KB*>(a.keys_out);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const uint32_t li = hbase + i * 16;
            if (li < num_valid) stcs(kout0 + tile_base + li, key[i]);
        }
        if constexpr (HAS_V) rs_copy_tile<VB>(a.vals_in, a.vals_out, tile_base, num_valid, tid, THREADS);
        return;
    }
    uint32_t dg[DIG ? ITEMS : 1];
    if constexpr (DIG) {
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const uint32_t li = hbase + i * 16;
            dg[i] = li < num_valid ? (uint32_t)__ldcs(a.digits + tile_base + li) : (RS_DIGITS - 1);
        }
    }
    auto digit_at = [&](int i, uint32_t li) -> uint32_t {
        if constexpr (DIG) return dg[i];
        else return li < num_valid ? digit_of<KB, KIND, DESC>(key[i], a.shift, a.mask) : (RS_DIGITS - 1);
    };
    // ---- values of a full tile: asynchronous copy into shared memory (input
    // order) that lands while the keys are ranked ------------------------------
    const VB* vin = reinterpret_cast<const VB*>(a.vals_in);
    bool v_staged = false;
    if constexpr (HAS_V) {
        v_staged = num_valid == (uint32_t)TILE && (reinterpret_cast<uintptr_t>(vin + tile_base) & 15) == 0;
        if (v_staged) {
            constexpr int CHUNKS = TILE * (int)sizeof(VB) / 16;
            const char* src = reinterpret_cast<const char*>(vin + tile_base);
            char* dst = reinterpret_cast<char*>(s_vals);
#pragma unroll
            for (int c = tid; c < CHUNKS; c += THREADS) cp_async16(dst + c * 16, src + c * 16);
            cp_async_commit();
        }
    }

    // ---- early counts: per-warp digit histogram of the tile -------------------
    uint32_t* wc = s_wc + (warp * 2 + half) * RS_DIGITS;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const uint32_t li = hbase + i * 16;
        const uint32_t d = digit_at(i, li);
        atomicAdd(wc + d, 1u);
    }
    __syncthreads();

    // ---- tile digit totals: publish at once, then tile-local digit offsets ---
    W* lb = reinterpret_cast<W*>(a.lookback);
    uint32_t total = 0;
    if (tid < RS_DIGITS) {
#pragma unroll
        for (int w = 0; w < RS_HALVES; ++w) total += s_wc[w * RS_DIGITS + tid];
        if (tile == 0)
            lb_store(lb + tid, F::INCL | (W)(a.bins[tid] + total));
        else
            lb_store(lb + tile * RS_DIGITS + tid, F::PART | (W)total);
    }
    // exclusive scan of the 256 totals (threads 0..255 = warps 0..7)
    uint32_t incl = total;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31 && warp < RS_DIGITS / 32) s_misc[1 + warp] = incl;
    __syncthreads();
    uint32_t off = 0;
    if (tid < RS_DIGITS) {
        for (int w = 0; w < warp; ++w) off += s_misc[1 + w];
        off += incl - total;
        // each half-warp's counter starts at the tile position of its first key of d
        uint32_t run = off;
#pragma unroll
        for (int w = 0; w < RS_HALVES; ++w) {
            const uint32_t c = s_wc[w * RS_DIGITS + tid];
            s_wc[w * RS_DIGITS + tid] = run;
            run += c;
        }
    }
    __syncthreads();

    // ---- per-digit look-back (warps 0..7; the other warps rank meanwhile) ----
    if (tid < RS_DIGITS) {
        W excl;
        if (tile == 0) {
            excl = a.bins[tid];
        } else {
            // Walk back over predecessors RS_LB_WINDOW at a time: the window's
            // words are loaded together (independent loads in flight), then
            // consumed nearest first until an inclusive word ends the walk.
            W acc = 0;
            int64_t pt = (int64_t)tile - 1;
            uint32_t spins = 0;
            const uint32_t limit = g_spin_limit;
            bool done = false;
            while (!done) {
                W w[RS_LB_WINDOW];
#pragma unroll
                for (int j = 0; j < RS_LB_WINDOW; ++j)
                    w[j] = pt - j >= 0 ? lb_load(lb + (uint64_t)(pt - j) * RS_DIGITS + tid) : F::INCL;
#pragma unroll
                for (int j = 0; j < RS_LB_WINDOW; ++j) {
                    if (done) break;
                    while ((w[j] & (F::PART | F::INCL)) == 0) {
                        if (++spins > limit) {
                            set_error(LCPP_ERR_LOOKBACK_TIMEOUT);
                            w[j] = F::INCL;  // give up: treat as resolved
                            break;
                        }
                        __nanosleep(spins < 16 ? 64 : 256);  // leave issue slots to the ranking warps
                        w[j] = lb_load(lb + (uint64_t)(pt - j) * RS_DIGITS + tid);
                    }
                    acc += w[j] & F::MASK;
                    if (w[j] & F::INCL) done = true;
                }
                pt -= RS_LB_WINDOW;
            }
            excl = acc;
            lb_store(lb + tile * RS_DIGITS + tid, F::INCL | (excl + total));
        }
        s_gbase[tid] = (uint32_t)excl - off;
    }

    // ---- stable rank: keys straight to their tile position in shared memory --
    const uint32_t lt = (1u << hl) - 1u;
    uint32_t pos[ITEMS];
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const uint32_t li = hbase + i * 16;
        const uint32_t d = digit_at(i, li);
        // Lanes of a half-warp holding the same digit set their bits in the
        // mask half of the word, read the word back (mask of peers and the
        // running position), and the highest peer writes the advanced
        // position with the mask cleared: three shared-memory accesses per key.
        atomicOr(wc + d, 1u << (16 + hl));
        __syncwarp();
        const uint32_t v = wc[d];
        const uint32_t peers = v >> 16;
        __syncwarp();
        pos[i] = (v & 0xFFFFu) + __popc(peers & lt);
        if ((peers >> hl) == 1u) wc[d] = (v & 0xFFFFu) + __popc(peers);
        __syncwarp();
        s_keys[pos[i]] = key[i];
        if constexpr (DIG) s_dig[pos[i]] = (uint8_t)d;
    }

    // ---- values into shared memory in digit order -----------------------------
    if constexpr (HAS_V) {
        VB val[ITEMS];
        if (v_staged) {
            cp_async_wait_all();
            __syncthreads();  // every thread's chunks have landed
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) val[i] = s_vals[hbase + i * 16];
            __syncthreads();  // staging fully read before it is overwritten
        } else {
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                const uint32_t li = hbase + i * 16;
                if (li < num_valid) val[i] = ldcs(vin + tile_base + li);
            }
        }
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const uint32_t li = hbase + i * 16;
            if (li < num_valid) s_vals[pos[i]] = val[i];
        }
    }
    __syncthreads();

    // ---- coalesced write-out ----------------------------------------------------
    KB* kout = reinterpret_cast<KB*>(a.keys_out);
    VB* vout = reinterpret_cast<VB*>(a.vals_out);
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const uint32_t idx = i * THREADS + tid;
        if (idx < num_valid) {
            const KB k = s_keys[idx];
            uint32_t d;
            if constexpr (DIG) d = s_dig[idx];
            else d = digit_of<KB, KIND, DESC>(k, a.shift, a.mask);
            const uint32_t g = s_gbase[d] + idx;
            stcs(kout + g, k);
            if constexpr (HAS_V) stcs(vout + g, s_vals[idx]);
        }
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct RsLayout {
    uint32_t passes;
    uint64_t tiles;
    size_t lb_word;
    size_t bins_off, ticket_off, lb_off, keys_off, vals_off, total, zero_bytes;
};

static RsLayout rs_layout(size_t ksize, size_t vsize, uint64_t n, uint32_t passes, bool dig = false) {
    RsLayout L{};
    const int items = rs_items_for(ksize, vsize, dig);
    L.passes = passes;
    L.tiles = ceil_div(n ? n : 1, (uint64_t)RS_THREADS * items);
    L.lb_word = n < (1ull << 30) ? 4 : 8;
    L.bins_off = 0;
    L.ticket_off = align_up(RS_MAX_PASSES * RS_DIGITS * 4, 256);
    L.lb_off = L.ticket_off + 256;
    L.keys_off = align_up(L.lb_off + (size_t)passes * L.tiles * RS_DIGITS * L.lb_word, 256);
    L.zero_bytes = L.lb_off + (size_t)passes * L.tiles * RS_DIGITS * L.lb_word;
    const bool alt = passes > 1;
    L.vals_off = align_up(L.keys_off + (alt ? n * ksize : 0), 256);
    L.total = align_up(L.vals_off + (alt ? n * vsize : 0), 256);
    return L;
}

static int key_kind(int dtype) {
    switch (dtype) {
        case LCPP_U32: case LCPP_U64: return 0;
        case LCPP_I32: case LCPP_I64: return 1;
        case LCPP_F32: case LCPP_F64: return 2;
        default: return -1;
    }
}

template <typename KB, typename VB, typename W, int KIND, bool DESC>
static lcpp_status rs_run(const RsLayout& L, const void* keys_in, void* keys_out, const void* vals_in,
                          void* vals_out, uint64_t n, uint32_t begin_bit, uint32_t end_bit, char* temp,
                          cudaStream_t s, const uint8_t* digits) {
    uint32_t* bins = (uint32_t*)(temp + L.bins_off);
    uint32_t* tickets = (uint32_t*)(temp + L.ticket_off);
    char* lb = temp + L.lb_off;
    {
        ProfScope ps("rs_memset", s);
        if (cudaMemsetAsync(temp, 0, L.zero_bytes, s) != cudaSuccess) return LCPP_ERR_CUDA;
    }

    const DeviceInfo di = device_info();
    {
        const uint64_t per_cta = (uint64_t)HISTC_THREADS * (16 / sizeof(KB)) * 4;
        uint64_t g = ceil_div(n, per_cta);
        const uint64_t cap = (uint64_t)di.sms;
        if (g > cap) g = cap;
        if (g == 0) g = 1;
        constexpr size_t hsmem = histc_smem_bytes<KB>();
        auto hk = rs_histogram_cols_kernel<KB, KIND, DESC>;
        if (cudaFuncSetAttribute(hk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hsmem) != cudaSuccess)
            return LCPP_ERR_CUDA;
        { ProfScope ps("rs_histogram", s);
        if (digits)
            rs_digit_hist_kernel<<<(unsigned)g, HISTC_THREADS, 0, s>>>(digits, n, bins);
        else
            hk<<<(unsigned)g, HISTC_THREADS, hsmem, s>>>((const KB*)keys_in, n, bins, begin_bit, end_bit, L.passes); }
        { ProfScope ps("rs_bins_scan", s);
        rs_bins_scan_kernel<<<L.passes, RS_DIGITS, 0, s>>>(bins, n, tickets + RS_MAX_PASSES); }
        count_launch(2);
    }
    const int threads = RS_THREADS;
    size_t smem;
    void (*kern)(RsPass);
    if (digits) {  // one pass over precomputed digits (only unsigned ascending instantiations)
        if constexpr (KIND == 0 && !DESC) {
            smem = rs_smem_bytes<KB, VB, RS_THREADS, true>();
            kern = rs_onesweep_kernel<KB, VB, W, 0, false, RS_THREADS, true>;
        } else {
            return LCPP_ERR_INVALID_ARG;
        }
    } else {
        smem = rs_smem_bytes<KB, VB, RS_THREADS>();
        kern = rs_onesweep_kernel<KB, VB, W, KIND, DESC, RS_THREADS>;
    }
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return LCPP_ERR_CUDA;

    const size_t ks = sizeof(KB);
    const size_t vs = std::is_same<VB, NoValue>::value ? 0 : sizeof(VB);
    void* kalt = temp + L.keys_off;
    void* valt = vs ? (void*)(temp + L.vals_off) : nullptr;
    const void* kcur = keys_in;
    const void* vcur = vals_in;
    for (uint32_t p = 0; p < L.passes; ++p) {
        // The pass whose distance to the last pass is even writes keys_out.
        const bool to_out = ((L.passes - 1 - p) & 1) == 0;
        RsPass a;
        a.keys_in = kcur;
        a.vals_in = vcur;
        a.keys_out = to_out ? keys_out : kalt;
        a.vals_out = vs ? (to_out ? vals_out : valt) : nullptr;
        a.n = n;
        a.shift = begin_bit + p * RS_BITS;
        const uint32_t nb = end_bit - a.shift < (uint32_t)RS_BITS ? end_bit - a.shift : (uint32_t)RS_BITS;
        a.mask = (1u << nb) - 1u;
        a.bins = bins + p * RS_DIGITS;
        a.lookback = lb + (size_t)p * L.tiles * RS_DIGITS * L.lb_word;
        a.ticket = tickets + p;
        a.identity = tickets + RS_MAX_PASSES + p;
        a.digits = digits;
        { ProfScope ps("rs_onesweep", s);
        kern<<<(unsigned)L.tiles, threads, smem, s>>>(a); }
        count_launch();
        kcur = a.keys_out;
        vcur = a.vals_out;
        (void)ks;
    }
    return check_launch();
}

template <typename KB, typename VB, int KIND>
static lcpp_status rs_dispatch_w(const RsLayout& L, bool desc, const void* ki, void* ko, const void* vi,
                                 void* vo, uint64_t n, uint32_t bb, uint32_t eb, char* t, cudaStream_t s,
                                 const uint8_t* sd) {
    if (L.lb_word == 4)
        return desc ? rs_run<KB, VB, uint32_t, KIND, true>(L, ki, ko, vi, vo, n, bb, eb, t, s, sd)
                    : rs_run<KB, VB, uint32_t, KIND, false>(L, ki, ko, vi, vo, n, bb, eb, t, s, sd);
    return desc ? rs_run<KB, VB, uint64_t, KIND, true>(L, ki, ko, vi, vo, n, bb, eb, t, s, sd)
                : rs_run<KB, VB, uint64_t, KIND, false>(L, ki, ko, vi, vo, n, bb, eb, t, s, sd);
}

template <typename KB, typename VB>
static lcpp_status rs_dispatch_kind(int kind, const RsLayout& L, bool desc, const void* ki, void* ko,
                                    const void* vi, void* vo, uint64_t n, uint32_t bb, uint32_t eb,
                                    char* t, cudaStream_t s, const uint8_t* sd) {
    switch (kind) {
        case 0: return rs_dispatch_w<KB, VB, 0>(L, desc, ki, ko, vi, vo, n, bb, eb, t, s, sd);
        case 1: return rs_dispatch_w<KB, VB, 1>(L, desc, ki, ko, vi, vo, n, bb, eb, t, s, sd);
        default: return rs_dispatch_w<KB, VB, 2>(L, desc, ki, ko, vi, vo, n, bb, eb, t, s, sd);
    }
}

static bool rs_bits(int key_dtype, int& begin_bit, int& end_bit, uint32_t& passes) {
    const int kbits = (int)lcpp_dtype_size(key_dtype) * 8;
    if (end_bit <= 0) end_bit = kbits;
    if (begin_bit < 0 || end_bit > kbits || begin_bit >= end_bit) return false;
    passes = (uint32_t)ceil_div((uint64_t)(end_bit - begin_bit), RS_BITS);
    return true;
}

}  // namespace lcpp

using namespace lcpp;

extern "C" size_t lcpp_radix_sort_temp_bytes(int key_dtype, int value_dtype, uint64_t n) {
    if (key_kind(key_dtype) < 0) return 0;
    const size_t ks = lcpp_dtype_size(key_dtype);
    const size_t vs = value_dtype == LCPP_NONE ? 0 : lcpp_dtype_size(value_dtype);
    if (value_dtype != LCPP_NONE && vs == 0) return 0;
    return rs_layout(ks, vs, n, (uint32_t)(ks * 8 / RS_BITS)).total;
}

namespace lcpp {
// Body of lcpp_radix_sort.  digits (device pointer or NULL): one pass that
// orders the items by a precomputed one-byte digit per item instead of key
// bits (stable); the multi-GPU sort partitions its shards by splitter bucket
// this way.  Needs begin_bit = 0, end_bit <= 8 and is served for unsigned
// ascending key views only (the caller passes keys as raw unsigned bits).
static lcpp_status rs_sort_impl(int key_dtype, int value_dtype, int descending,
                                const void* keys_in, void* keys_out,
                                const void* values_in, void* values_out, uint64_t n,
                                int begin_bit, int end_bit,
                                void* temp, size_t temp_bytes, void* stream, const uint8_t* digits) {
    const int kind = key_kind(key_dtype);
    if (kind < 0) return LCPP_ERR_INVALID_ARG;
    const size_t ks = lcpp_dtype_size(key_dtype);
    const size_t vs = value_dtype == LCPP_NONE ? 0 : lcpp_dtype_size(value_dtype);
    if (value_dtype != LCPP_NONE && vs == 0) return LCPP_ERR_INVALID_ARG;
    if (n >= (1ull << 32)) return LCPP_ERR_INVALID_ARG;
    uint32_t passes = 0;
    if (!rs_bits(key_dtype, begin_bit, end_bit, passes)) return LCPP_ERR_INVALID_ARG;
    if (n == 0) return LCPP_OK;
    if (!keys_in || !keys_out || (vs && (!values_in || !values_out))) return LCPP_ERR_INVALID_ARG;
    // Temp is sized for a full-width sort; fewer bits need no more.
    if (!temp || temp_bytes < lcpp_radix_sort_temp_bytes(key_dtype, value_dtype, n)) return LCPP_ERR_TEMP_TOO_SMALL;
    const RsLayout L = rs_layout(ks, vs, n, passes, digits != nullptr);
    cudaStream_t s = (cudaStream_t)stream;
    char* t = (char*)temp;
    const bool desc = descending != 0;
    const uint32_t bb = (uint32_t)begin_bit, eb = (uint32_t)end_bit;
    const uint8_t* sd = digits;
    if (ks == 4) {
        if (vs == 0) return rs_dispatch_kind<uint32_t, NoValue>(kind, L, desc, keys_in, keys_out, nullptr, nullptr, n, bb, eb, t, s, sd);
        if (vs == 4) return rs_dispatch_kind<uint32_t, uint32_t>(kind, L, desc, keys_in, keys_out, values_in, values_out, n, bb, eb, t, s, sd);
        return rs_dispatch_kind<uint32_t, uint64_t>(kind, L, desc, keys_in, keys_out, values_in, values_out, n, bb, eb, t, s, sd);
    }
    if (vs == 0) return rs_dispatch_kind<uint64_t, NoValue>(kind, L, desc, keys_in, keys_out, nullptr, nullptr, n, bb, eb, t, s, sd);
    if (vs == 4) return rs_dispatch_kind<uint64_t, uint32_t>(kind, L, desc, keys_in, keys_out, values_in, values_out, n, bb, eb, t, s, sd);
    return rs_dispatch_kind<uint64_t, uint64_t>(kind, L, desc, keys_in, keys_out, values_in, values_out, n, bb, eb, t, s, sd);
}
}  // namespace lcpp

extern "C" lcpp_status lcpp_radix_sort(int key_dtype, int value_dtype, int descending,
                                       const void* keys_in, void* keys_out,
                                       const void* values_in, void* values_out, uint64_t n,
                                       int begin_bit, int end_bit,
                                       void* temp, size_t temp_bytes, void* stream) {
    return rs_sort_impl(key_dtype, value_dtype, descending, keys_in, keys_out, values_in, values_out, n,
                        begin_bit, end_bit, temp, temp_bytes, stream, nullptr);
}

// ---------------------------------------------------------------------------
// Digit-run boundaries of keys already ordered by one 8-bit digit.
// ---------------------------------------------------------------------------
namespace lcpp {

template <typename KB, int KIND>
__global__ void rs_bucket_starts_kernel(const KB* keys, uint64_t n, uint32_t shift, uint64_t* starts) {
    const uint32_t b = threadIdx.x;  // 256 threads: first index whose digit >= b
    uint64_t lo = 0, hi = n;
    while (lo < hi) {
        const uint64_t mid = (lo + hi) >> 1;
        const uint32_t d = (uint32_t)(ordered_bits<KB, KIND, false>(keys[mid]) >> shift) & 0xFFu;
        if (d < b) lo = mid + 1; else hi = mid;
    }
    starts[b] = lo;
    if (b == 0) starts[RS_DIGITS] = n;
}

}  // namespace lcpp

extern "C" lcpp_status lcpp_radix_bucket_starts(int key_dtype, const void* keys, uint64_t n, int bit_start,
                                                uint64_t* starts, void* stream) {
    const int kind = key_kind(key_dtype);
    const int kbits = (int)lcpp_dtype_size(key_dtype) * 8;
    if (kind < 0 || !starts || (n && !keys) || bit_start < 0 || bit_start + 8 > kbits) return LCPP_ERR_INVALID_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    auto go = [&](auto kb) -> lcpp_status {
        using KB = decltype(kb);
        const KB* k = (const KB*)keys;
        switch (kind) {
            case 0: rs_bucket_starts_kernel<KB, 0><<<1, RS_DIGITS, 0, s>>>(k, n, bit_start, starts); break;
            case 1: rs_bucket_starts_kernel<KB, 1><<<1, RS_DIGITS, 0, s>>>(k, n, bit_start, starts); break;
            default: rs_bucket_starts_kernel<KB, 2><<<1, RS_DIGITS, 0, s>>>(k, n, bit_start, starts); break;
        }
        count_launch();
        return check_launch();
    };
    return kbits == 32 ? go((uint32_t)0) : go((uint64_t)0);
}
