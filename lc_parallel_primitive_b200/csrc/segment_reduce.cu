// DeviceSegmentReduce for sm_100a with segment-length-aware mapping.
//
// Reference behaviour followed: segment_reduce_array_recursive
// (src/lcpp/device/device_segment_reduce.h:353-381) and its kernel
// (src/lcpp/device/details/segment_reduce.h:43-86): out[s] = init (+)
// reduce(in[begin[s]..end[s])), empty segment -> init; fixed-size variant
// (details/segment_reduce.h:98-164).  The reference runs one 256-thread CTA
// per segment; at 2^20 segments of ~128 items most of those threads idle.
//
// B200 mapping (with a temp buffer from lcpp_segment_reduce_temp_bytes the
// flat item-tiled path below runs; these two kernels serve calls with less
// temp, fixed-size segments, and offsets that are not monotone):
//  * Kernel A: one warp per segment (8 segments per 256-thread CTA), lanes
//    read consecutive elements (4 independent loads in flight per lane).  A
//    segment longer than SEG_LONG is not reduced here: its id is appended to a
//    work list in temp.
//  * Kernel B: persistent CTAs (2 per SM) take long segments from that list
//    and reduce each with a whole 512-thread CTA using 128-bit loads.
// Each segment is reduced by exactly one warp or one CTA in a fixed order, so
// float results do not depend on scheduling.
#include "common.cuh"
#include <algorithm>

namespace lcpp {

constexpr int SEG_A_THREADS = 256;
constexpr int SEG_A_WARPS = SEG_A_THREADS / 32;
constexpr int SEG_B_THREADS = 512;
constexpr int SEG_B_CTAS_PER_SM = 2;
constexpr uint64_t SEG_LONG = 4096;
constexpr size_t SEG_HDR = 256;

template <typename Op, typename T, bool FIXED>
__global__ void __launch_bounds__(SEG_A_THREADS)
seg_warp_kernel(const T* __restrict__ in, T* __restrict__ out, uint64_t num_segments,
                const uint32_t* __restrict__ begin, const uint32_t* __restrict__ end,
                uint64_t seg_size, T init, unsigned int* long_count, uint32_t* long_list) {
    const int lane = threadIdx.x & 31;
    const uint64_t s = (uint64_t)blockIdx.x * SEG_A_WARPS + (threadIdx.x >> 5);
    if (s >= num_segments) return;
    uint64_t b, e;
    if (FIXED) {
        b = s * seg_size;
        e = b + seg_size;
    } else {
        b = __ldg(begin + s);
        e = __ldg(end + s);
        if (e < b) e = b;
    }
    if (long_list && e - b > SEG_LONG) {
        if (lane == 0) long_list[atomicAdd(long_count, 1u)] = (uint32_t)s;
        return;
    }
    T acc = Op::template identity<T>();
    uint64_t i = b + lane;
    for (; i + 96 < e; i += 128) {
        const T x0 = ldcs(in + i), x1 = ldcs(in + i + 32), x2 = ldcs(in + i + 64), x3 = ldcs(in + i + 96);
        acc = Op::template apply<T>(acc, Op::template apply<T>(Op::template apply<T>(x0, x1), Op::template apply<T>(x2, x3)));
    }
    for (; i < e; i += 32) acc = Op::template apply<T>(acc, ldcs(in + i));
    acc = warp_reduce<Op>(acc);
    if (lane == 0) out[s] = Op::template apply<T>(init, acc);
}

template <typename Op, typename T, bool FIXED>
__global__ void __launch_bounds__(SEG_B_THREADS)
seg_block_kernel(const T* __restrict__ in, T* __restrict__ out,
                 const uint32_t* __restrict__ begin, const uint32_t* __restrict__ end,
                 uint64_t seg_size, T init, const unsigned int* long_count,
                 const uint32_t* long_list, uint64_t fixed_count) {
    constexpr int VEC = 16 / sizeof(T);
    __shared__ T s_warp[SEG_B_THREADS / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t count = FIXED ? fixed_count : (uint64_t)*long_count;
    for (uint64_t j = blockIdx.x; j < count; j += gridDim.x) {
        const uint64_t s = FIXED ? j : long_list[j];
        uint64_t b, e;
        if (FIXED) {
            b = s * seg_size;
            e = b + seg_size;
        } else {
            b = begin[s];
            e = end[s];
        }
        T acc = Op::template identity<T>();
        // scalar head to a 16-byte boundary, 128-bit body, scalar tail
        const uint64_t mis = (reinterpret_cast<uintptr_t>(in + b) & 15) / sizeof(T);
        uint64_t head = mis ? VEC - mis : 0;
        if (head > e - b) head = e - b;
        if (threadIdx.x < head) acc = Op::template apply<T>(acc, in[b + threadIdx.x]);
        const uint64_t vb = b + head;
        const uint64_t nvec = (e - vb) / VEC;
        const uint4* v = reinterpret_cast<const uint4*>(in + vb);
        uint64_t k = threadIdx.x;
        for (; k + 3 * SEG_B_THREADS < nvec; k += 4 * SEG_B_THREADS) {
            uint4 q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q[u] = ld_stream(v + k + u * SEG_B_THREADS);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const T* x = reinterpret_cast<const T*>(&q[u]);
#pragma unroll
                for (int t = 0; t < VEC; ++t) acc = Op::template apply<T>(acc, x[t]);
            }
        }
        for (; k < nvec; k += SEG_B_THREADS) {
            const uint4 q = ld_stream(v + k);
            const T* x = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int t = 0; t < VEC; ++t) acc = Op::template apply<T>(acc, x[t]);
        }
        const uint64_t t0 = vb + nvec * VEC;
        if (t0 + threadIdx.x < e) acc = Op::template apply<T>(acc, in[t0 + threadIdx.x]);
        acc = warp_reduce<Op>(acc);
        if (lane == 0) s_warp[warp] = acc;
        __syncthreads();
        if (warp == 0) {
            acc = lane < SEG_B_THREADS / 32 ? s_warp[lane] : Op::template identity<T>();
            acc = warp_reduce<Op>(acc);
            if (lane == 0) out[s] = Op::template apply<T>(init, acc);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Flat item-tiled path (offsets that are monotone: begin[s] <= end[s] <=
// begin[s+1]; CSR offsets are).  The work is split by ITEMS, not segments,
// so every load is an independent 16-byte copy and HBM stays busy whatever
// the segment lengths:
//  * segf_partition_kernel (one thread per segment): first segment of every
//    SEGF_BYTES tile (the first whose end is past the tile start), the tile
//    count, and a flag if the offsets are not monotone or the tiles do not fit
//    the temp buffer;
//  * segf_main_kernel (persistent): a tile's items (and its segments'
//    offsets) land in shared memory by cp.async.  When the tile's segments
//    are contiguous, each thread reduces 32 consecutive items split at
//    segment heads and the pieces are joined by a segmented scan; otherwise
//    one warp per segment piece reduces it (lane-strided, then a shuffle
//    tree).  A segment wholly inside the tile is written at once; a
//    segment that crosses the tile's right edge leaves its piece in carry[c];
//    one that enters from the left leaves it in head[c];
//  * segf_fixup_kernel (one warp per tile with a head piece): out[s] = init
//    (+) carries of the tiles the segment crosses (lane-strided, shuffle tree)
//    (+) head piece.  Every combination order is fixed, so float results do
//    not depend on scheduling;
//    When the flag is set the same kernel reduces one warp per segment
//    instead (the fallback).  The three kernels are chained by programmatic
//    dependent launch, so each one's launch overlaps the previous kernel.
// ---------------------------------------------------------------------------
constexpr int SEGF_THREADS = 256;
constexpr int SEGF_WARPS = SEGF_THREADS / 32;
constexpr int SEGF_BYTES = 32768;                  // items per tile = SEGF_BYTES / sizeof(T)
constexpr int SEGF_CHUNK = 512;                    // segment offsets staged per round
constexpr int SEGF_CTAS_PER_SM = 4;
constexpr uint32_t SEGF_NONE = 0xffffffffu;

struct SegfHdr {
    unsigned int flag;    // nonzero: use the fallback
    unsigned int ntiles;
};

template <typename T>
struct SegfTemp {
    SegfHdr* hdr;
    uint32_t* first;      // [cap + 1] first segment per tile
    T* carry;             // [cap]
    uint32_t* carry_seg;  // [cap]
    T* head;              // [cap]
    uint32_t* head_seg;   // [cap]
    uint64_t cap;
};

template <typename T>
static size_t segf_bytes_per_tile() { return 2 * sizeof(T) + 3 * sizeof(uint32_t); }

template <typename T>
static SegfTemp<T> segf_carve(void* temp, size_t bytes) {
    SegfTemp<T> t{};
    char* p = (char*)temp;
    t.hdr = (SegfHdr*)p;
    const size_t avail = bytes > SEG_HDR + 1024 ? bytes - SEG_HDR - 1024 : 0;
    t.cap = avail / segf_bytes_per_tile<T>();
    p += SEG_HDR;
    t.carry = (T*)p; p += align_up(t.cap * sizeof(T), 8);
    t.head = (T*)p; p += align_up(t.cap * sizeof(T), 8);
    t.first = (uint32_t*)p; p += (t.cap + 1) * 4;
    t.carry_seg = (uint32_t*)p; p += t.cap * 4;
    t.head_seg = (uint32_t*)p;
    return t;
}

template <typename T>
__global__ void __launch_bounds__(256)
segf_partition_kernel(const uint32_t* __restrict__ begin, const uint32_t* __restrict__ end, uint64_t S,
                      SegfTemp<T> t) {
    constexpr uint64_t TI = SEGF_BYTES / sizeof(T);
    // the tile kernel may be scheduled now; its griddepcontrol.wait still waits for this grid's writes
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    const uint64_t e = end[s], b = begin[s];
    const uint64_t pe = s ? end[s - 1] : 0;
    if (b > e || (s && pe > b)) atomicOr(&t.hdr->flag, 1u);
    // tiles whose start c*TI lies in [pe, e) begin inside segment s (or its gap)
    for (uint64_t c = (pe + TI - 1) / TI; c * TI < e; ++c) {
        if (c >= t.cap) { atomicOr(&t.hdr->flag, 2u); break; }
        t.first[c] = (uint32_t)s;
    }
    if (s == S - 1) {
        const uint64_t nt = (e + TI - 1) / TI;
        if (nt == 0 || nt > t.cap) atomicOr(&t.hdr->flag, 2u);  // no items: the fallback writes init
        else { t.hdr->ntiles = (unsigned)nt; t.first[nt] = (uint32_t)S; }
    }
}

// Shared-memory layout of a staged tile: row r (the items of thread r on the
// item-parallel path, 128 bytes) holds 16-byte chunk j at position j ^ (r & 7),
// so the eight rows a quarter-warp reads fall on different banks.
template <typename T>
__device__ __forceinline__ uint32_t segf_slot(uint32_t i) {
    constexpr uint32_t EPC = 16 / sizeof(T);
    const uint32_t c = i / EPC, r = c >> 3, j = c & 7;
    return (((r << 3) | (j ^ (r & 7))) * EPC) + (i % EPC);
}
__device__ __forceinline__ uint32_t segf_chunk_slot(uint32_t c) { return ((c >> 3) << 3) | ((c & 7) ^ ((c >> 3) & 7)); }

// Reduce items [lo, hi) of the staged tile (tile-relative) with one warp.
template <typename Op, typename T>
__device__ __forceinline__ T segf_warp_piece(const T* tile, uint32_t lo, uint32_t hi, int lane) {
    T acc = Op::template identity<T>();
    for (uint32_t i = lo + lane; i < hi; i += 32) acc = Op::template apply<T>(acc, tile[segf_slot<T>(i)]);
    return warp_reduce<Op>(acc);
}

// (has a segment head, value) pairs of the item-parallel path: the value runs
// from the last head seen (or from the start) to the end of the span.
template <typename Op, typename T>
__device__ __forceinline__ void segf_combine(bool& f, T& v, bool fn, T vn) {  // (f, v) = (f, v) then (fn, vn)
    v = fn ? vn : Op::template apply<T>(v, vn);
    f = f || fn;
}

template <typename Op, typename T>
__global__ void __launch_bounds__(SEGF_THREADS, SEGF_CTAS_PER_SM)
segf_main_kernel(const T* __restrict__ in, T* __restrict__ out, const uint32_t* __restrict__ begin,
                 const uint32_t* __restrict__ end, uint64_t S, T init, SegfTemp<T> t) {
    constexpr uint32_t TI = SEGF_BYTES / sizeof(T);
    __shared__ __align__(16) T s_tile[TI];
    __shared__ uint32_t s_b[SEGF_CHUNK], s_e[SEGF_CHUNK];
    constexpr uint32_t SEGF_HBW = TI / 32;  // head bitmap words
    __shared__ uint32_t s_hb[SEGF_HBW];
    __shared__ bool s_wf[SEGF_WARPS];
    __shared__ T s_wv[SEGF_WARPS];
    __shared__ uint32_t s_wk[SEGF_WARPS];
    extern __shared__ uint16_t s_segat[];  // [TI] segment (relative to lo) starting at each head position
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the partition kernel has completed
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (t.hdr->flag) return;
    const uint64_t ntiles = t.hdr->ntiles;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool vec = (reinterpret_cast<uintptr_t>(in) & 15) == 0;
    const uint64_t last_end = end[S - 1];  // the last tile ends at the last segment end
    uint64_t nlo = 0, nhi = 0;              // segment range of the next tile, loaded one tile ahead
    if (blockIdx.x < ntiles) {
        nlo = blockIdx.x ? t.first[blockIdx.x] : 0;
        nhi = t.first[blockIdx.x + 1];
    }
    for (uint64_t c = blockIdx.x; c < ntiles; c += gridDim.x) {
        const uint64_t base = c * TI;
        const uint32_t cnt = (uint32_t)min((uint64_t)TI, last_end - base);
        const uint64_t lo = nlo;
        const uint64_t hi = nhi;  // exclusive; segment hi may cross the right edge
        const uint64_t m = hi - lo;
        const bool has_next = hi < S;      // segment hi starts in this tile or at its end
        bool fast = m + 1 <= SEGF_CHUNK;   // uniform over the CTA
        const uint32_t M = (uint32_t)m + (has_next ? 1u : 0u);
        __syncthreads();  // previous tile fully consumed
        // the tile, and (item-parallel path) the offsets of its segments, in one cp.async group
        if (vec && cnt == TI) {
            constexpr int CH = SEGF_BYTES / 16;
            for (int k = threadIdx.x; k < CH; k += SEGF_THREADS)
                cp_async16(reinterpret_cast<char*>(s_tile) + segf_chunk_slot(k) * 16,
                           reinterpret_cast<const char*>(in + base) + k * 16);
        } else {
            for (uint32_t k = threadIdx.x; k < cnt; k += SEGF_THREADS) s_tile[segf_slot<T>(k)] = in[base + k];
        }
        if (fast) {
            for (uint32_t k = threadIdx.x; k < M; k += SEGF_THREADS) {
                cp_async4(s_b + k, begin + lo + k);
                cp_async4(s_e + k, end + lo + k);
            }
            for (uint32_t k = threadIdx.x; k < SEGF_HBW; k += SEGF_THREADS) s_hb[k] = 0u;
        }
        cp_async_commit();
        if (c + gridDim.x < ntiles) {
            nlo = t.first[c + gridDim.x];
            nhi = t.first[c + gridDim.x + 1];
        }
        if (threadIdx.x == 0) { t.carry_seg[c] = SEGF_NONE; t.head_seg[c] = SEGF_NONE; }
        cp_async_wait_all();
        __syncthreads();
        // ---- item-parallel path: contiguous segments, at most SEGF_CHUNK - 1 owned.
        // Thread r reduces its IPL consecutive items, splitting them at segment
        // heads (a bitmap of the owned segments' begins); the pieces are joined
        // across threads by a segmented scan of (has head, value) pairs.
        if (fast) {
            bool ok = true;
            for (uint32_t k = threadIdx.x; k < M; k += SEGF_THREADS) {
                const uint64_t b = s_b[k], e = s_e[k];
                if (k == 0 ? b > base : b != s_e[k - 1]) ok = false;
                if (e > b && b >= base && b < base + cnt) {
                    atomicOr(&s_hb[(uint32_t)(b - base) >> 5], 1u << ((b - base) & 31));
                    s_segat[b - base] = (uint16_t)k;
                }
            }
            fast = __syncthreads_and(ok);
        }
        if (fast) {
            // piece of owned segment kk (index relative to lo) is complete: out, or the head piece
            auto emit = [&](uint32_t kk, T v) {
                if (s_b[kk] >= base) out[lo + kk] = Op::template apply<T>(init, v);
                else { t.head[c] = v; t.head_seg[c] = (uint32_t)(lo + kk); }
            };
            for (uint32_t k = threadIdx.x; k < (uint32_t)m; k += SEGF_THREADS)
                if (s_e[k] == s_b[k]) out[lo + k] = init;  // empty segments
            constexpr uint32_t IPL = TI / SEGF_THREADS;  // 32 (4-byte) or 16 (8-byte) items per thread
            constexpr uint32_t EPC = 16 / sizeof(T);
            const uint32_t r = threadIdx.x, p0 = r * IPL;
            T x[IPL];
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) {
                const uint4 qv = reinterpret_cast<const uint4*>(s_tile)[(r << 3) | (j ^ (r & 7))];
                const T* e = reinterpret_cast<const T*>(&qv);
#pragma unroll
                for (uint32_t u = 0; u < EPC; ++u) x[j * EPC + u] = e[u];
            }
            const uint32_t hb = IPL == 32 ? s_hb[r] : (s_hb[r >> 1] >> (16 * (r & 1))) & 0xFFFFu;
            const uint32_t nv = cnt > p0 ? min(IPL, cnt - p0) : 0u;
            T cur = Op::template identity<T>(), pre = cur;
            bool hh = false;
            uint32_t ks = 0;  // segment (relative to lo) of the current piece once a head was seen
            // a head closes the piece before it; a piece begun at a head inside
            // this thread's items started in the tile, so it goes straight to out
            auto step = [&](uint32_t j) {
                const bool hd = (hb >> j) & 1u;
                if (hd) {
                    if (hh) out[lo + ks] = Op::template apply<T>(init, cur);
                    else pre = cur;
                    ks = s_segat[p0 + j];
                    hh = true;
                }
                cur = hd ? x[j] : Op::template apply<T>(cur, x[j]);
            };
            if (nv == IPL) {
#pragma unroll
                for (uint32_t j = 0; j < IPL; ++j) step(j);
            } else {
#pragma unroll
                for (uint32_t j = 0; j < IPL; ++j)
                    if (j < nv) step(j);
            }
            // warp-inclusive segmented scan of (hh, cur, ks): value and segment of the open piece
            bool fi = hh;
            T vi = cur;
            uint32_t ki = ks;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const bool fy = __shfl_up_sync(0xffffffffu, fi, o);
                const T vy = __shfl_up_sync(0xffffffffu, vi, o);
                const uint32_t ky = __shfl_up_sync(0xffffffffu, ki, o);
                if (lane >= o) {
                    if (!fi) { vi = Op::template apply<T>(vy, vi); ki = ky; }
                    fi = fi || fy;
                }
            }
            bool fx = __shfl_up_sync(0xffffffffu, fi, 1);
            T vx = __shfl_up_sync(0xffffffffu, vi, 1);
            uint32_t kx = __shfl_up_sync(0xffffffffu, ki, 1);
            if (lane == 0) { fx = false; vx = Op::template identity<T>(); kx = 0; }
            if (lane == 31) { s_wf[warp] = fi; s_wv[warp] = vi; s_wk[warp] = ki; }
            __syncthreads();
            bool fc = false;  // no head before: the open piece belongs to segment lo
            T vc = Op::template identity<T>();
            uint32_t kc = 0;
            for (int w = 0; w < warp; ++w) {
                if (s_wf[w]) { vc = s_wv[w]; kc = s_wk[w]; fc = true; }
                else vc = Op::template apply<T>(vc, s_wv[w]);
            }
            if (fx) { vc = vx; kc = kx; fc = true; }
            else vc = Op::template apply<T>(vc, vx);
            // vc, kc: the piece open where this thread's items begin
            // the first head closes the piece before it (empty when the head is at tile position 0)
            if (hh && !(p0 == 0 && (hb & 1u))) emit(kc, Op::template apply<T>(vc, pre));
            if (threadIdx.x == SEGF_THREADS - 1) {  // the piece open at the tile end
                if (hh) { vc = cur; kc = ks; }
                else vc = Op::template apply<T>(vc, cur);
                if (has_next && c + 1 < ntiles && kc == M - 1) {  // segment hi crosses the right edge
                    t.carry[c] = vc;
                    t.carry_seg[c] = (uint32_t)hi;
                } else {
                    emit(kc, vc);
                }
            }
            continue;
        }
        // segments owned by this tile (end inside it), in chunks of offsets
        for (uint64_t s0 = lo; s0 < hi; s0 += SEGF_CHUNK) {
            const uint32_t m = (uint32_t)min((uint64_t)SEGF_CHUNK, hi - s0);
            __syncthreads();
            for (uint32_t k = threadIdx.x; k < m; k += SEGF_THREADS) { s_b[k] = begin[s0 + k]; s_e[k] = end[s0 + k]; }
            __syncthreads();
            for (uint32_t k = warp; k < m; k += SEGF_WARPS) {
                const uint64_t b = s_b[k], e = s_e[k];
                const uint32_t plo = b > base ? (uint32_t)(b - base) : 0u;
                const uint32_t phi = (uint32_t)(e - base);
                const T v = segf_warp_piece<Op, T>(s_tile, plo, phi > plo ? phi : plo, lane);
                if (lane == 0) {
                    if (b >= base || e == b) out[s0 + k] = Op::template apply<T>(init, v);
                    else { t.head[c] = v; t.head_seg[c] = (uint32_t)(s0 + k); }
                }
            }
        }
        // the segment crossing the right edge
        if (warp == 0 && c + 1 < ntiles && hi < S) {
            const uint64_t b = begin[hi];
            if (b < base + TI) {
                const uint32_t plo = b > base ? (uint32_t)(b - base) : 0u;
                const T v = segf_warp_piece<Op, T>(s_tile, plo, TI, lane);
                if (lane == 0) { t.carry[c] = v; t.carry_seg[c] = (uint32_t)hi; }
            }
        }
    }
}

// Fix-up, or (flag set by the partition kernel) the per-segment fallback.
template <typename Op, typename T>
__global__ void __launch_bounds__(256)
segf_fixup_kernel(const T* __restrict__ in, T* __restrict__ out, uint64_t S, const uint32_t* __restrict__ begin,
                  const uint32_t* __restrict__ end, T init, SegfTemp<T> t) {
    constexpr uint64_t TI = SEGF_BYTES / sizeof(T);
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the tile kernel has completed
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    const uint64_t gw = (uint64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t.hdr->flag) {  // offsets not monotone or tiles beyond the temp: one warp per segment
        for (uint64_t sg = gw; sg < S; sg += warps) {
            uint64_t b = begin[sg], e = end[sg];
            if (e < b) e = b;
            T acc = Op::template identity<T>();
            for (uint64_t i = b + lane; i < e; i += 32) acc = Op::template apply<T>(acc, ldcs(in + i));
            acc = warp_reduce<Op>(acc);
            if (lane == 0) out[sg] = Op::template apply<T>(init, acc);
        }
        return;
    }
    const uint64_t ntiles = t.hdr->ntiles;
    for (uint64_t c = gw; c < ntiles; c += warps) {
        const uint32_t s = t.head_seg[c];
        if (s == SEGF_NONE) continue;
        const uint64_t c0 = begin[s] / TI;
        T acc = Op::template identity<T>();
        for (uint64_t k = c0 + lane; k < c; k += 32) acc = Op::template apply<T>(acc, t.carry[k]);
        acc = warp_reduce<Op>(acc);
        if (lane == 0) out[s] = Op::template apply<T>(Op::template apply<T>(init, acc), t.head[c]);
    }
}

// Launch with programmatic dependent launch: the kernel may start while the
// previous kernel on the stream runs and waits for it with griddepcontrol.wait.
template <typename... KArgs, typename... Args>
static cudaError_t segf_launch_pdl(void (*k)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t s,
                                   Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

template <typename Op, typename T>
static lcpp_status segf_launch(const void* in, void* out, uint64_t S, const uint32_t* begin, const uint32_t* end,
                               void* temp, size_t temp_bytes, cudaStream_t s) {
    const T init = Op::template identity<T>();
    const SegfTemp<T> t = segf_carve<T>(temp, temp_bytes);
    const DeviceInfo di = device_info();
    if (cudaMemsetAsync(t.hdr, 0, sizeof(SegfHdr), s) != cudaSuccess) return LCPP_ERR_CUDA;
    { ProfScope ps("seg_partition", s);
    segf_partition_kernel<T><<<(unsigned)ceil_div(S, 256), 256, 0, s>>>(begin, end, S, t); }
    constexpr int SEGAT = (SEGF_BYTES / sizeof(T)) * sizeof(uint16_t);
    if (cudaFuncSetAttribute(segf_main_kernel<Op, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SEGAT) != cudaSuccess)
        return LCPP_ERR_CUDA;
    { ProfScope ps("seg_flat", s);
    if (segf_launch_pdl(segf_main_kernel<Op, T>, (unsigned)(di.sms * SEGF_CTAS_PER_SM), SEGF_THREADS, SEGAT, s,
                        (const T*)in, (T*)out, begin, end, S, init, t) != cudaSuccess)
        return LCPP_ERR_CUDA; }
    { ProfScope ps("seg_fixup", s);
    if (segf_launch_pdl(segf_fixup_kernel<Op, T>, (unsigned)(di.sms * 8), 256, 0, s, (const T*)in, (T*)out, S, begin,
                        end, init, t) != cudaSuccess)
        return LCPP_ERR_CUDA; }
    count_launch(3);
    return check_launch();
}

template <typename Op, typename T>
static lcpp_status seg_launch(const void* in, void* out, uint64_t S, const uint32_t* begin,
                              const uint32_t* end, uint64_t seg_size, bool fixed, void* temp,
                              cudaStream_t s) {
    const T init = Op::template identity<T>();
    const DeviceInfo di = device_info();
    if (fixed) {
        if (seg_size > SEG_LONG) {
            uint64_t g = (uint64_t)di.sms * SEG_B_CTAS_PER_SM * 4;
            if (g > S) g = S;
            seg_block_kernel<Op, T, true><<<(unsigned)g, SEG_B_THREADS, 0, s>>>(
                (const T*)in, (T*)out, nullptr, nullptr, seg_size, init, nullptr, nullptr, S);
        } else {
            seg_warp_kernel<Op, T, true><<<(unsigned)ceil_div(S, SEG_A_WARPS), SEG_A_THREADS, 0, s>>>(
                (const T*)in, (T*)out, S, nullptr, nullptr, seg_size, init, nullptr, nullptr);
        }
        count_launch();
        return check_launch();
    }
    if (!temp) {  // no work list: every segment is reduced by one warp
        ProfScope ps("seg_warp", s);
        seg_warp_kernel<Op, T, false><<<(unsigned)ceil_div(S, SEG_A_WARPS), SEG_A_THREADS, 0, s>>>(
            (const T*)in, (T*)out, S, begin, end, 0, init, nullptr, nullptr);
        count_launch();
        return check_launch();
    }
    unsigned int* cnt = (unsigned int*)temp;
    uint32_t* list = (uint32_t*)((char*)temp + SEG_HDR);
    if (cudaMemsetAsync(cnt, 0, sizeof(unsigned int), s) != cudaSuccess) return LCPP_ERR_CUDA;
    { ProfScope ps("seg_warp", s);
    seg_warp_kernel<Op, T, false><<<(unsigned)ceil_div(S, SEG_A_WARPS), SEG_A_THREADS, 0, s>>>(
        (const T*)in, (T*)out, S, begin, end, 0, init, cnt, list); }
    ProfScope ps("seg_block", s);
    uint64_t g = (uint64_t)di.sms * SEG_B_CTAS_PER_SM;
    seg_block_kernel<Op, T, false><<<(unsigned)g, SEG_B_THREADS, 0, s>>>(
        (const T*)in, (T*)out, begin, end, 0, init, cnt, list, 0);
    count_launch(2);
    return check_launch();
}

template <typename T>
static lcpp_status seg_op(int op, const void* in, void* out, uint64_t S, const uint32_t* begin,
                          const uint32_t* end, uint64_t seg_size, bool fixed, void* temp, cudaStream_t s,
                          size_t flat_bytes = 0) {
    if (flat_bytes) {
        switch (op) {
            case LCPP_OP_SUM: return segf_launch<OpSum, T>(in, out, S, begin, end, temp, flat_bytes, s);
            case LCPP_OP_MIN: return segf_launch<OpMin, T>(in, out, S, begin, end, temp, flat_bytes, s);
            default: return segf_launch<OpMax, T>(in, out, S, begin, end, temp, flat_bytes, s);
        }
    }
    switch (op) {
        case LCPP_OP_SUM: return seg_launch<OpSum, T>(in, out, S, begin, end, seg_size, fixed, temp, s);
        case LCPP_OP_MIN: return seg_launch<OpMin, T>(in, out, S, begin, end, seg_size, fixed, temp, s);
        default: return seg_launch<OpMax, T>(in, out, S, begin, end, seg_size, fixed, temp, s);
    }
}

}  // namespace lcpp

using namespace lcpp;

// Temp of the flat path for num_items items (state of every tile plus a spare
// tile), or at least the long-segment work list of the per-segment path.
static size_t segf_temp_bytes(size_t es, uint64_t num_items) {
    const uint64_t tiles = ceil_div(num_items, SEGF_BYTES / es) + 1;
    return SEG_HDR + 1024 + tiles * (2 * es + 3 * sizeof(uint32_t)) + 256;
}

extern "C" size_t lcpp_segment_reduce_temp_bytes(int dtype, uint64_t num_items, uint64_t num_segments) {
    const size_t es = lcpp_dtype_size(dtype);
    if (!es) return 0;
    const size_t list = SEG_HDR + align_up((num_segments ? num_segments : 1) * sizeof(uint32_t), 256);
    const size_t flat = segf_temp_bytes(es, num_items);
    return list > flat ? list : flat;
}

extern "C" lcpp_status lcpp_segment_reduce(int op, int dtype, const void* in, void* out,
                                           uint64_t num_segments, const uint32_t* begin_offsets,
                                           const uint32_t* end_offsets, void* temp,
                                           size_t temp_bytes, void* stream) {
    if (op < 0 || op > 2 || !lcpp_dtype_size(dtype)) return LCPP_ERR_INVALID_ARG;
    if (num_segments == 0) return LCPP_OK;
    if (!out || !begin_offsets || !end_offsets || num_segments > 0xffffffffull) return LCPP_ERR_INVALID_ARG;
    // With temp for at least one tile the flat item-tiled path runs (it
    // checks on the device that the offsets are monotone and that all tiles
    // fit, else reduces one warp per segment).  With less temp: the
    // per-segment path, with (or, without room for it, without) the
    // long-segment work list.
    const size_t es = lcpp_dtype_size(dtype);
    const size_t flat = temp && temp_bytes >= segf_temp_bytes(es, 1) ? temp_bytes : 0;
    if (!flat && (!temp || temp_bytes < SEG_HDR + align_up(num_segments * sizeof(uint32_t), 256))) temp = nullptr;
    return dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        return seg_op<T>(op, in, out, num_segments, begin_offsets, end_offsets, 0, false, temp,
                         (cudaStream_t)stream, flat);
    });
}

extern "C" lcpp_status lcpp_segment_reduce_fixed(int op, int dtype, const void* in, void* out,
                                                 uint64_t num_segments, uint64_t segment_size,
                                                 void* stream) {
    if (op < 0 || op > 2 || !lcpp_dtype_size(dtype)) return LCPP_ERR_INVALID_ARG;
    if (num_segments == 0) return LCPP_OK;
    if (!out || (!in && segment_size)) return LCPP_ERR_INVALID_ARG;
    return dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        return seg_op<T>(op, in, out, num_segments, nullptr, nullptr, segment_size, true, nullptr,
                         (cudaStream_t)stream);
    });
}
