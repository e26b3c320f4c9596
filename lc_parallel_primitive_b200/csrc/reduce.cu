// DeviceReduce for sm_100a: one grid-stride kernel with 128-bit streaming
// loads and a last-CTA-done combine, so a full reduction is one launch (plus a
// 4-byte memset of the ticket counter).
//
// Reference behaviour followed: DeviceReduce::Reduce / reduce_array_recursive
// (src/lcpp/device/device_reduce.h:131-147, 396-460), AgentReduce tile
// consumption (src/lcpp/agent/agent_reduce.h:59-157) and the single-tile
// finalisation out = reduce_op(init, aggregate)
// (src/lcpp/device/details/reduce.h:214-237).  The reference reduces level by
// level (3 launches + a copy at n = 2^24); here the partials of one level are
// combined in-kernel by the last CTA to finish, in a fixed order, so float
// results are deterministic for a given n and GPU.
#include "common.cuh"
#include <type_traits>

namespace lcpp {

constexpr int REDUCE_THREADS = 512;
constexpr int REDUCE_CTAS_PER_SM = 8;
constexpr int REDUCE_UNROLL = 4;   // independent 16-byte loads in flight per thread
constexpr int REDUCE_MAX_GRID = 148 * 16;

template <typename Op, typename T>
__device__ __forceinline__ T block_reduce(T v, T* s_warp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_reduce<Op>(v);
    if (lane == 0) s_warp[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : Op::template identity<T>();
        v = warp_reduce<Op>(v);
    }
    return v;  // valid in warp 0
}

// Element transforms of TransformReduce (the reference takes a DSL lambda,
// device_reduce.h:331-348; a C ABI carries one of these instead).  Integer
// square and negate wrap modulo 2^bits.  Each takes the kernel's runtime
// factor k (-1 for negate, unused otherwise): negation is a multiply by a
// value the compiler cannot see, because on this toolchain a max reduction
// over compiler-visible negations (0 - x, whatever its spelling) came out
// with some elements not negated.
struct XfIdentity { template <typename T> static __device__ __forceinline__ T apply(T x, T) { return x; } };
struct XfSquare {
    template <typename T> static __device__ __forceinline__ T apply(T x, T) {
        if constexpr (std::is_floating_point<T>::value) return x * x;
        else {
            using U = typename Unsigned<T>::type;
            return (T)((U)x * (U)x);
        }
    }
};
struct XfAbs {
    template <typename T> static __device__ __forceinline__ T apply(T x, T) {
        if constexpr (std::is_unsigned<T>::value) return x;
        else if constexpr (std::is_floating_point<T>::value) return x < T(0) ? -x : x;  // -0 and NaN kept
        else {
            using U = typename Unsigned<T>::type;
            return x < T(0) ? (T)(U(0) - (U)x) : x;
        }
    }
};
struct XfNegate {
    template <typename T> static __device__ __forceinline__ T apply(T x, T k) {
        if constexpr (std::is_floating_point<T>::value) return x * k;
        else {
            using U = typename Unsigned<T>::type;
            return (T)((U)x * (U)k);
        }
    }
};

// Accumulate the 16-byte vector `q` (VEC elements of T) into acc.
template <typename Op, typename T, int VEC, typename Xf = XfIdentity>
__device__ __forceinline__ T fold_vec(T acc, const uint4& q, T k = T(0)) {
    const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc = Op::template apply<T>(acc, Xf::template apply<T>(e[i], k));
    return acc;
}

template <typename Op, typename T, typename Xf = XfIdentity>
__global__ void __launch_bounds__(REDUCE_THREADS)
reduce_kernel(const T* __restrict__ in, uint64_t n, T* __restrict__ partials,
              unsigned int* __restrict__ ticket, T* __restrict__ out, T init, T k = T(0)) {
    constexpr int VEC = 16 / sizeof(T);
    __shared__ T s_warp[REDUCE_THREADS / 32];
    __shared__ bool s_last;

    T acc = Op::template identity<T>();
    // Scalar head up to the first 16-byte boundary, vector body, scalar tail.
    const uint64_t mis = (reinterpret_cast<uintptr_t>(in) & 15) / sizeof(T);
    uint64_t head = mis ? (uint64_t)(VEC - mis) : 0;
    if (head > n) head = n;
    const uint64_t gtid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t gstride = (uint64_t)gridDim.x * blockDim.x;
    if (gtid < head) acc = Op::template apply<T>(acc, Xf::template apply<T>(in[gtid], k));

    const uint4* vin = reinterpret_cast<const uint4*>(in + head);
    const uint64_t nvec = (n - head) / VEC;
    uint64_t i = gtid;
    for (; i + (REDUCE_UNROLL - 1) * gstride < nvec; i += REDUCE_UNROLL * gstride) {
        uint4 q[REDUCE_UNROLL];
#pragma unroll
        for (int u = 0; u < REDUCE_UNROLL; ++u) q[u] = ld_stream(vin + i + u * gstride);
#pragma unroll
        for (int u = 0; u < REDUCE_UNROLL; ++u) acc = fold_vec<Op, T, VEC, Xf>(acc, q[u], k);
    }
    if (i < nvec) {  // the last partial round: its loads are issued together, not one round trip each
        uint4 q[REDUCE_UNROLL - 1];
#pragma unroll
        for (int u = 0; u < REDUCE_UNROLL - 1; ++u)
            if (i + u * gstride < nvec) q[u] = ld_stream(vin + i + u * gstride);
#pragma unroll
        for (int u = 0; u < REDUCE_UNROLL - 1; ++u)
            if (i + u * gstride < nvec) acc = fold_vec<Op, T, VEC, Xf>(acc, q[u], k);
    }
    const uint64_t tail0 = head + nvec * VEC;
    if (tail0 + gtid < n) acc = Op::template apply<T>(acc, Xf::template apply<T>(in[tail0 + gtid], k));

    acc = block_reduce<Op>(acc, s_warp);
    if (!ticket) {  // two-kernel form: reduce_final_kernel combines the partials
        if (threadIdx.x == 0) partials[blockIdx.x] = acc;
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        return;
    }
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = acc;
        __threadfence();
        s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Last CTA: combine the partials in a fixed order (thread-strided, then tree).
    T v = Op::template identity<T>();
    for (unsigned int b = threadIdx.x; b < gridDim.x; b += blockDim.x)
        v = Op::template apply<T>(v, __ldcg(partials + b));
    __syncthreads();  // s_warp reuse
    v = block_reduce<Op>(v, s_warp);
    if (threadIdx.x == 0) out[0] = Op::template apply<T>(init, v);
}

// Second kernel of the two-kernel form, launched with programmatic dependent
// launch so that its launch overlaps the partial-sum kernel:
// griddepcontrol.wait blocks until that kernel has completed and its writes
// are visible.  One CTA combines the partials in a fixed order.
template <typename Op, typename T>
__global__ void __launch_bounds__(REDUCE_THREADS)
reduce_final_kernel(const T* __restrict__ partials, unsigned int count, T* __restrict__ out, T init) {
    __shared__ T s_warp[REDUCE_THREADS / 32];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    T v = Op::template identity<T>();
    for (unsigned int b = threadIdx.x; b < count; b += blockDim.x) v = Op::template apply<T>(v, partials[b]);
    v = block_reduce<Op>(v, s_warp);
    if (threadIdx.x == 0) out[0] = Op::template apply<T>(init, v);
}

template <typename Op, typename T, typename Xf = XfIdentity>
static lcpp_status reduce_two_kernels(const T* in, uint64_t n, T* part, T* out, unsigned grid, cudaStream_t s,
                                      T init = Op::template identity<T>(), T k = T(0)) {
    reduce_kernel<Op, T, Xf><<<grid, REDUCE_THREADS, 0, s>>>(in, n, part, nullptr, out, Op::template identity<T>(), k);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(REDUCE_THREADS);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, reduce_final_kernel<Op, T>, (const T*)part, grid, out, init) != cudaSuccess)
        return LCPP_ERR_CUDA;
    count_launch(2);
    return check_launch();
}

static bool reduce_use_pdl() {
    static const bool on = [] {
        const char* e = getenv("LCPP_REDUCE_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

static unsigned int reduce_grid(uint64_t n, int elem_size) {
    const DeviceInfo d = device_info();
    const uint64_t per_cta = (uint64_t)REDUCE_THREADS * (16 / elem_size) * REDUCE_UNROLL;
    uint64_t g = ceil_div(n ? n : 1, per_cta);
    uint64_t cap = (uint64_t)d.sms * REDUCE_CTAS_PER_SM;
    if (cap > REDUCE_MAX_GRID) cap = REDUCE_MAX_GRID;
    if (g > cap) g = cap;
    return (unsigned int)(g ? g : 1);
}

}  // namespace lcpp

using namespace lcpp;

extern "C" size_t lcpp_reduce_temp_bytes(int dtype, uint64_t n) {
    (void)n;
    size_t es = lcpp_dtype_size(dtype);
    if (!es || dtype == LCPP_NONE) return 0;
    // [ticket u32 | pad to 256][partials: one per CTA of the largest grid]
    return 256 + align_up((size_t)REDUCE_MAX_GRID * es, 256);
}

extern "C" lcpp_status lcpp_reduce(int op, int dtype, const void* in, void* out, uint64_t n,
                                   void* temp, size_t temp_bytes, void* stream) {
    if (!out || (!in && n) || (op < 0 || op > 2)) return LCPP_ERR_INVALID_ARG;
    const size_t need = lcpp_reduce_temp_bytes(dtype, n);
    if (!need) return LCPP_ERR_INVALID_ARG;
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned int* ticket = (unsigned int*)temp;
    void* partials = (char*)temp + 256;
    const bool pdl = reduce_use_pdl();
    if (!pdl && cudaMemsetAsync(ticket, 0, sizeof(unsigned int), s) != cudaSuccess) return LCPP_ERR_CUDA;
    return dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        const unsigned int grid = reduce_grid(n, sizeof(T));
        const T* pin = (const T*)in;
        T* pout = (T*)out;
        T* part = (T*)partials;
        ProfScope ps("reduce", s);
        if (pdl) {
            switch (op) {
                case LCPP_OP_SUM: return reduce_two_kernels<OpSum, T>(pin, n, part, pout, grid, s);
                case LCPP_OP_MIN: return reduce_two_kernels<OpMin, T>(pin, n, part, pout, grid, s);
                default: return reduce_two_kernels<OpMax, T>(pin, n, part, pout, grid, s);
            }
        }
        switch (op) {
            case LCPP_OP_SUM:
                reduce_kernel<OpSum, T><<<grid, REDUCE_THREADS, 0, s>>>(pin, n, part, ticket, pout, OpSum::identity<T>());
                break;
            case LCPP_OP_MIN:
                reduce_kernel<OpMin, T><<<grid, REDUCE_THREADS, 0, s>>>(pin, n, part, ticket, pout, OpMin::identity<T>());
                break;
            default:
                reduce_kernel<OpMax, T><<<grid, REDUCE_THREADS, 0, s>>>(pin, n, part, ticket, pout, OpMax::identity<T>());
                break;
        }
        count_launch();
        return check_launch();
    });
}

extern "C" lcpp_status lcpp_transform_reduce(int op, int transform, int dtype, const void* in, void* out,
                                             uint64_t n, const void* init, void* temp, size_t temp_bytes,
                                             void* stream) {
    if (!out || (!in && n) || op < 0 || op > 2 || transform < 0 || transform > 3) return LCPP_ERR_INVALID_ARG;
    const size_t need = lcpp_reduce_temp_bytes(dtype, n);
    if (!need) return LCPP_ERR_INVALID_ARG;
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    cudaStream_t s = (cudaStream_t)stream;
    return dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        const unsigned int grid = reduce_grid(n, sizeof(T));
        const T* pin = (const T*)in;
        T* pout = (T*)out;
        T* part = (T*)((char*)temp + 256);
        ProfScope ps("reduce", s);
        auto go = [&](auto opv) -> lcpp_status {
            using Op = decltype(opv);
            const T iv = init ? *(const T*)init : Op::template identity<T>();
            switch (transform) {
                case LCPP_XF_IDENTITY: return reduce_two_kernels<Op, T, XfIdentity>(pin, n, part, pout, grid, s, iv);
                case LCPP_XF_SQUARE: return reduce_two_kernels<Op, T, XfSquare>(pin, n, part, pout, grid, s, iv);
                case LCPP_XF_ABS: return reduce_two_kernels<Op, T, XfAbs>(pin, n, part, pout, grid, s, iv);
                default: return reduce_two_kernels<Op, T, XfNegate>(pin, n, part, pout, grid, s, iv, (T)-1);
            }
        };
        switch (op) {
            case LCPP_OP_SUM: return go(OpSum{});
            case LCPP_OP_MIN: return go(OpMin{});
            default: return go(OpMax{});
        }
    });
}
