// DeviceScan for sm_100a: single-pass prefix sum with decoupled look-back
// (Merrill & Garland 2016), the algorithm of the reference's ScanModule
// (src/lcpp/device/details/scan.h:59-147) and TilePrefixCallbackOp
// (src/lcpp/device/details/single_pass_scan_operator.h:138-251).
//
// B200 design:
//  * 32768-item tiles (1024 threads x 32 items), 128-bit streaming loads and
//    stores; each warp owns 1024 contiguous items, each thread eight 16-byte
//    vectors at a 512-byte stride, so every load/store instruction is one
//    fully coalesced 512-byte warp access.
//  * Thread-local scans, then shuffle scans per vector, then a 32-entry scan of
//    warp totals: no shared-memory transpose.
//  * Tile descriptors are single 64-bit words {status:32 | value:32} written
//    and read with relaxed device-scope atomics, so value and status can never
//    be seen out of step (the reference writes them separately with no fence,
//    single_pass_scan_operator.h:81-93).
//  * Tile ids come from an atomic ticket, so a tile only waits on tiles that
//    already started (forward progress without co-residency assumptions).
//  * Every wait is bounded: after g_spin_limit polls the tile latches
//    LCPP_ERR_LOOKBACK_TIMEOUT and carries on (no trap, no hang).
#include "common.cuh"

namespace lcpp {

constexpr int SCAN_THREADS = 1024;
constexpr int SCAN_WARPS = SCAN_THREADS / 32;
constexpr int SCAN_VECS = 8;                       // 16-byte vectors per thread
constexpr size_t SCAN_HDR = 256;                   // ticket counter + padding
// Items per 16-byte vector and per tile of scan_kernel (32768 4-byte or
// 16384 8-byte items).
template <typename T> __host__ __device__ constexpr int scan_vec_items() { return 16 / (int)sizeof(T); }
template <typename T> __host__ __device__ constexpr int scan_tile_items() { return SCAN_THREADS * SCAN_VECS * scan_vec_items<T>(); }
constexpr int SCAN_TILE = SCAN_THREADS * SCAN_VECS * 4;  // 4-byte types
// Smallest tile of any scan kernel (the pipelined kernel's 32 KiB tiles)
// sizes the descriptor arrays: 8192 4-byte or 4096 8-byte items.
constexpr int SCAN_DESC_TILE_BYTES = 32768;
constexpr int SCAN_DESC_TILE = SCAN_DESC_TILE_BYTES / 4;

template <typename Op, typename T>
static lcpp_status scan_pipe_launch(bool inclusive, const T* in, T* out, uint64_t n, const T* carry_in, T init,
                                    unsigned int* ticket, void* desc, cudaStream_t s);

constexpr uint64_t ST_PARTIAL = 1ull << 32;
constexpr uint64_t ST_INCLUSIVE = 2ull << 32;

template <typename T> __device__ __forceinline__ uint32_t to_bits(T v) { return __float_as_uint((float)v); }
template <> __device__ __forceinline__ uint32_t to_bits<uint32_t>(uint32_t v) { return v; }
template <> __device__ __forceinline__ uint32_t to_bits<int32_t>(int32_t v) { return (uint32_t)v; }
template <typename T> __device__ __forceinline__ T from_bits(uint32_t b) { return (T)__uint_as_float(b); }
template <> __device__ __forceinline__ uint32_t from_bits<uint32_t>(uint32_t b) { return b; }
template <> __device__ __forceinline__ int32_t from_bits<int32_t>(uint32_t b) { return (int32_t)b; }

// Tile descriptors of the look-back.  status: 0 not yet published,
// 1 partial (tile aggregate), 2 inclusive (prefix through the tile).
//  * 4-byte values: one 64-bit word {status:32 | value:32} per tile, written
//    and read with relaxed device-scope accesses, so value and status are
//    always seen together (the reference writes them as separate volatile
//    stores with no fence, single_pass_scan_operator.h:81-93).
//  * 8-byte values: two 64-bit words per tile, {status:32 | low half:32} and
//    {status:32 | high half:32}, written and read with relaxed device-scope
//    accesses (the two loads are independent, so both are in flight at once).
//    Each status is written once per tile with one value, so when both words
//    show the same status their halves belong to the same value; a reader
//    that sees different statuses (a write in between) treats the tile as not
//    yet published and loads it again.
template <typename T, bool WIDE = (sizeof(T) == 8)>
struct ScanDesc;

template <typename T>
struct ScanDesc<T, false> {
    uint64_t* w;
    static size_t bytes(uint64_t tiles) { return align_up(tiles * sizeof(uint64_t), 256); }
    static ScanDesc carve(void* p, uint64_t) { return ScanDesc{(uint64_t*)p}; }
    __device__ __forceinline__ void partial(int64_t t, T v) const { st_relaxed_u64(w + t, ST_PARTIAL | to_bits<T>(v)); }
    __device__ __forceinline__ void inclusive(int64_t t, T v) const { st_relaxed_u64(w + t, ST_INCLUSIVE | to_bits<T>(v)); }
    __device__ __forceinline__ uint32_t load(int64_t t, T& v) const {
        const uint64_t d = ld_relaxed_u64(w + t);
        v = from_bits<T>((uint32_t)d);
        return (uint32_t)(d >> 32);
    }
};

template <typename T>
struct ScanDesc<T, true> {
    uint64_t* w;  // [tiles][2]
    static size_t bytes(uint64_t tiles) { return align_up(tiles * 16, 256); }
    static ScanDesc carve(void* p, uint64_t) { return ScanDesc{(uint64_t*)p}; }
    __device__ __forceinline__ void put(int64_t t, uint64_t st, T v) const {
        uint64_t b;
        memcpy(&b, &v, 8);
        st_relaxed_u64(w + 2 * t, st | (b & 0xFFFFFFFFull));
        st_relaxed_u64(w + 2 * t + 1, st | (b >> 32));
    }
    __device__ __forceinline__ void partial(int64_t t, T v) const { put(t, ST_PARTIAL, v); }
    __device__ __forceinline__ void inclusive(int64_t t, T v) const { put(t, ST_INCLUSIVE, v); }
    __device__ __forceinline__ uint32_t load(int64_t t, T& v) const {
        const uint64_t d0 = ld_relaxed_u64(w + 2 * t);
        const uint64_t d1 = ld_relaxed_u64(w + 2 * t + 1);
        const uint32_t s0 = (uint32_t)(d0 >> 32);
        if (s0 != (uint32_t)(d1 >> 32)) return 0u;  // halves of different writes: not yet published
        const uint64_t b = (d1 << 32) | (d0 & 0xFFFFFFFFull);
        memcpy(&v, &b, 8);
        return s0;
    }
};

__device__ __forceinline__ void backoff(uint32_t it) {
    if (it > 64) __nanosleep(it < 1024 ? 32 : 128);
}

// Warp-wide look-back over descriptors[0..tile): returns the sum of the
// aggregates of all preceding tiles (same value in every lane).  Lane L
// inspects tile (window_end - L); windows of 32 move towards tile 0 until an
// inclusive descriptor is found.
template <typename Op, typename T, typename D>
__device__ T lookback_warp(const D& desc, int64_t tile) {
    const int lane = threadIdx.x & 31;
    const uint32_t limit = g_spin_limit;
    T acc = Op::template identity<T>();
    int64_t p = tile - 1 - lane;
    uint32_t spins = 0;
    while (true) {
        T v = Op::template identity<T>();
        uint32_t st = p >= 0 ? desc.load(p, v) : 2u;
        while (__any_sync(0xffffffffu, st == 0)) {
            if (++spins > limit) {
                if (lane == 0) set_error(LCPP_ERR_LOOKBACK_TIMEOUT);
                return warp_reduce<Op>(acc);
            }
            backoff(spins);
            if (st == 0) st = desc.load(p, v);
        }
        const uint32_t incl = __ballot_sync(0xffffffffu, st == 2);
        if (incl) {
            const int first = __ffs(incl) - 1;
            if (lane > first) v = Op::template identity<T>();
            return Op::template apply<T>(acc, warp_reduce<Op>(v));
        }
        acc = Op::template apply<T>(acc, warp_reduce<Op>(v));
        p -= 32;
    }
}

// Warp 0 of a tile: publish the tile aggregate, resolve the exclusive prefix,
// publish the inclusive value.  Returns the exclusive prefix in every lane.
template <typename Op, typename T, typename D>
__device__ __forceinline__ T tile_prefix(const D& desc, int64_t tile, T aggregate, T carry) {
    const int lane = threadIdx.x & 31;
    if (tile == 0) {
        if (lane == 0) desc.inclusive(0, Op::template apply<T>(carry, aggregate));
        return carry;
    }
    if (lane == 0) desc.partial(tile, aggregate);
    const T excl = lookback_warp<Op, T>(desc, tile);
    if (lane == 0) desc.inclusive(tile, Op::template apply<T>(excl, aggregate));
    return excl;
}

template <typename Op, typename T, bool INCLUSIVE, typename D = ScanDesc<T>>
__global__ void __launch_bounds__(SCAN_THREADS, 1)
scan_kernel(const T* in, T* out, uint64_t n, const T* carry_in, T init,
            unsigned int* ticket, D desc) {
    constexpr int V = scan_vec_items<T>();
    constexpr int WARP_ITEMS = 32 * SCAN_VECS * V;
    constexpr int TILE = scan_tile_items<T>();
    __shared__ unsigned int s_tile;
    __shared__ T s_warp[SCAN_WARPS];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1u);
    __syncthreads();
    const int64_t tile = s_tile;
    const uint64_t tile_base = (uint64_t)tile * TILE;
    const uint64_t base = tile_base + (uint64_t)warp * WARP_ITEMS + lane * V;
    const bool vec_ok = tile_base + TILE <= n &&
                        ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;

    T x[SCAN_VECS][V];
    if (vec_ok) {
#pragma unroll
        for (int j = 0; j < SCAN_VECS; ++j) {
            const uint4 q = ld_stream(reinterpret_cast<const uint4*>(in + base + j * 32 * V));
            const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int k = 0; k < V; ++k) x[j][k] = e[k];
        }
    } else {
#pragma unroll
        for (int j = 0; j < SCAN_VECS; ++j)
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const uint64_t i = base + j * 32 * V + k;
                x[j][k] = i < n ? in[i] : Op::template identity<T>();
            }
    }

    // Thread-local inclusive scans, then one warp scan per vector.
    T pre[SCAN_VECS];  // exclusive prefix of each vector within the warp
    T carry = Op::template identity<T>();
#pragma unroll
    for (int j = 0; j < SCAN_VECS; ++j) {
#pragma unroll
        for (int k = 1; k < V; ++k) x[j][k] = Op::template apply<T>(x[j][k - 1], x[j][k]);
        T incl = x[j][V - 1];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const T y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl = Op::template apply<T>(y, incl);
        }
        T excl = __shfl_up_sync(0xffffffffu, incl, 1);
        if (lane == 0) excl = Op::template identity<T>();
        pre[j] = Op::template apply<T>(carry, excl);
        carry = Op::template apply<T>(carry, __shfl_sync(0xffffffffu, incl, 31));
    }
    if (lane == 0) s_warp[warp] = carry;
    __syncthreads();

    if (warp == 0) {
        const T wt = lane < SCAN_WARPS ? s_warp[lane] : Op::template identity<T>();
        T incl = wt;
#pragma unroll
        for (int o = 1; o < SCAN_WARPS; o <<= 1) {
            const T y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl = Op::template apply<T>(y, incl);
        }
        const T aggregate = __shfl_sync(0xffffffffu, incl, SCAN_WARPS - 1);
        const T c0 = carry_in ? *carry_in : init;
        const T block_excl = tile_prefix<Op, T>(desc, tile, aggregate, c0);
        __syncwarp();
        // All 32 lanes take part in the shuffle; only SCAN_WARPS store.
        T wex = __shfl_up_sync(0xffffffffu, incl, 1);
        if (lane == 0) wex = Op::template identity<T>();
        if (lane < SCAN_WARPS) s_warp[lane] = Op::template apply<T>(block_excl, wex);
    }
    __syncthreads();
    const T wbase = s_warp[warp];

    if (vec_ok) {
#pragma unroll
        for (int j = 0; j < SCAN_VECS; ++j) {
            const T b = Op::template apply<T>(wbase, pre[j]);
            T r[V];
            if (INCLUSIVE) {
#pragma unroll
                for (int k = 0; k < V; ++k) r[k] = Op::template apply<T>(b, x[j][k]);
            } else {
                r[0] = b;
#pragma unroll
                for (int k = 1; k < V; ++k) r[k] = Op::template apply<T>(b, x[j][k - 1]);
            }
            __stcs(reinterpret_cast<uint4*>(out + base + j * 32 * V), *reinterpret_cast<const uint4*>(r));
        }
    } else {
#pragma unroll
        for (int j = 0; j < SCAN_VECS; ++j) {
            const T b = Op::template apply<T>(wbase, pre[j]);
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const uint64_t i = base + j * 32 * V + k;
                if (i < n) out[i] = INCLUSIVE ? Op::template apply<T>(b, x[j][k]) : (k ? Op::template apply<T>(b, x[j][k - 1]) : b);
            }
        }
    }
}

// ---- stand-alone look-back (unit hooks) -----------------------------------
__global__ void lookback_tiles_kernel(const uint32_t* agg, uint32_t* excl_out, uint32_t* incl_out,
                                      unsigned int* ticket, uint64_t* desc) {
    __shared__ unsigned int s_tile;
    if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1u);
    __syncwarp();
    const int64_t tile = s_tile;
    const uint32_t a = agg[tile];
    const uint32_t e = tile_prefix<OpSum, uint32_t>(ScanDesc<uint32_t>{desc}, tile, a, 0u);
    if (threadIdx.x == 0) {
        excl_out[tile] = e;
        incl_out[tile] = e + a;
    }
}

__global__ void lookback_probe_kernel(const uint64_t* desc, int64_t tile, uint32_t* excl_out) {
    const uint32_t e = lookback_warp<OpSum, uint32_t>(ScanDesc<uint32_t>{const_cast<uint64_t*>(desc)}, tile);
    if (threadIdx.x == 0) *excl_out = e;
}

}  // namespace lcpp

using namespace lcpp;

static size_t scan_desc_tiles(size_t es, uint64_t n) { return ceil_div(n ? n : 1, SCAN_DESC_TILE_BYTES / es); }

extern "C" size_t lcpp_scan_temp_bytes(int dtype, uint64_t n) {
    const size_t es = lcpp_dtype_size(dtype);
    if (!es || dtype == LCPP_NONE) return 0;
    const uint64_t tiles = scan_desc_tiles(es, n);
    return SCAN_HDR + (es == 4 ? ScanDesc<uint32_t>::bytes(tiles) : ScanDesc<uint64_t>::bytes(tiles));
}

// Shared body of the scan entry points: op in {SUM, MIN, MAX}; the device
// carry (multi-GPU) or, without one, the host value *init seeds tile 0.
static lcpp_status scan_impl(int kind, int op, int dtype, const void* in, void* out, uint64_t n,
                             const void* carry_in, const void* init, void* temp, size_t temp_bytes, void* stream) {
    if ((kind != LCPP_SCAN_EXCLUSIVE && kind != LCPP_SCAN_INCLUSIVE) || op < 0 || op > 2 || (n && (!in || !out)))
        return LCPP_ERR_INVALID_ARG;
    const size_t need = lcpp_scan_temp_bytes(dtype, n);
    if (!need) return LCPP_ERR_INVALID_ARG;
    if (n == 0) return LCPP_OK;
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    const size_t es = lcpp_dtype_size(dtype);
    const uint64_t desc_tiles = scan_desc_tiles(es, n);
    if (desc_tiles > 0xffffffffull) return LCPP_ERR_INVALID_ARG;
    const bool aligned = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned int* ticket = (unsigned int*)temp;
    void* desc_mem = (char*)temp + SCAN_HDR;
    auto go_op = [&](auto zero, auto opv) -> lcpp_status {
        using T = decltype(zero);
        using Op = decltype(opv);
        using D = ScanDesc<T>;
        const uint64_t tiles = aligned ? desc_tiles : ceil_div(n, scan_tile_items<T>());
        // zero the ticket and the descriptors (one 64-bit word per tile, two for 8-byte values)
        const size_t zero_bytes = SCAN_HDR + tiles * (sizeof(T) == 4 ? 8 : 16);
        if (cudaMemsetAsync(temp, 0, zero_bytes, s) != cudaSuccess) return LCPP_ERR_CUDA;
        const D desc = D::carve(desc_mem, desc_tiles);
        const T iv = init ? *(const T*)init : Op::template identity<T>();
        const T* ci = (const T*)carry_in;
        ProfScope ps("scan", s);
        if (aligned)  // pipelined persistent kernel (scan_pipe.cu)
            return scan_pipe_launch<Op, T>(kind == LCPP_SCAN_INCLUSIVE, (const T*)in, (T*)out, n, ci, iv, ticket,
                                           desc_mem, s);
        if (kind == LCPP_SCAN_INCLUSIVE)
            scan_kernel<Op, T, true><<<(unsigned)tiles, SCAN_THREADS, 0, s>>>((const T*)in, (T*)out, n, ci, iv, ticket, desc);
        else
            scan_kernel<Op, T, false><<<(unsigned)tiles, SCAN_THREADS, 0, s>>>((const T*)in, (T*)out, n, ci, iv, ticket, desc);
        count_launch();
        return check_launch();
    };
    auto go = [&](auto zero) -> lcpp_status {
        switch (op) {
            case LCPP_OP_SUM: return go_op(zero, OpSum{});
            case LCPP_OP_MIN: return go_op(zero, OpMin{});
            default: return go_op(zero, OpMax{});
        }
    };
    return dispatch_dtype(dtype, go);
}

extern "C" lcpp_status lcpp_scan_carry(int kind, int dtype, const void* in, void* out, uint64_t n,
                                       const void* carry_in, void* temp, size_t temp_bytes, void* stream) {
    return scan_impl(kind, LCPP_OP_SUM, dtype, in, out, n, carry_in, nullptr, temp, temp_bytes, stream);
}

extern "C" lcpp_status lcpp_scan_op(int kind, int op, int dtype, const void* in, void* out, uint64_t n,
                                    const void* init, void* temp, size_t temp_bytes, void* stream) {
    return scan_impl(kind, op, dtype, in, out, n, nullptr, init, temp, temp_bytes, stream);
}

extern "C" lcpp_status lcpp_scan(int kind, int dtype, const void* in, void* out, uint64_t n,
                                 void* temp, size_t temp_bytes, void* stream) {
    return lcpp_scan_carry(kind, dtype, in, out, n, nullptr, temp, temp_bytes, stream);
}

extern "C" size_t lcpp_lookback_temp_bytes(uint64_t num_tiles) {
    return SCAN_HDR + align_up((num_tiles ? num_tiles : 1) * sizeof(uint64_t), 256);
}

extern "C" lcpp_status lcpp_lookback_tiles(const uint32_t* aggregates, uint32_t* exclusive_out,
                                           uint32_t* inclusive_out, uint64_t num_tiles,
                                           void* temp, size_t temp_bytes, void* stream) {
    if (num_tiles == 0) return LCPP_OK;
    if (!aggregates || !exclusive_out || !inclusive_out || num_tiles > 0x7fffffffull) return LCPP_ERR_INVALID_ARG;
    if (!temp || temp_bytes < lcpp_lookback_temp_bytes(num_tiles)) return LCPP_ERR_TEMP_TOO_SMALL;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(temp, 0, SCAN_HDR + num_tiles * 8, s) != cudaSuccess) return LCPP_ERR_CUDA;  // 64-bit words
    lookback_tiles_kernel<<<(unsigned)num_tiles, 32, 0, s>>>(aggregates, exclusive_out, inclusive_out,
                                                             (unsigned int*)temp,
                                                             (uint64_t*)((char*)temp + SCAN_HDR));
    count_launch();
    return check_launch();
}

extern "C" lcpp_status lcpp_lookback_probe(const uint64_t* descriptors, uint64_t tile,
                                           uint32_t* exclusive_out, void* stream) {
    if (!descriptors || !exclusive_out) return LCPP_ERR_INVALID_ARG;
    lookback_probe_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(descriptors, (int64_t)tile, exclusive_out);
    count_launch();
    return check_launch();
}
