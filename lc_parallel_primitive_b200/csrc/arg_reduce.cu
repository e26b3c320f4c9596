// ArgMin / ArgMax over a whole array and over segments.
//
// Reference behaviour followed: DeviceReduce::ArgMin/ArgMax
// (src/lcpp/device/device_reduce.h:187-275) and DeviceSegmentReduce::ArgMin/
// ArgMax (src/lcpp/device/device_segment_reduce.h:197-349), which reduce
// (index, value) pairs with ArgMinOp / ArgMaxOp
// (src/lcpp/common/thread_operators.h:19-47):
//   ArgMin keeps b over a when b.value < a.value, or equal values and b.index < a.index;
//   ArgMax keeps b over a when b.value > a.value, or equal values and b.index > a.index.
// Both are order-independent, so the result does not depend on the reduction
// tree: ArgMin returns the first minimum, ArgMax the last maximum.  Segment
// indices are relative to the segment's begin (arg_assign,
// src/lcpp/device/details/segment_reduce.h:198-215).  An empty input or
// segment gives {index 1, max() for ArgMin / lowest() for ArgMax}.
//
// B200 mapping: the index is implied by the position, so no (index, value)
// array is built (the reference materialises one, arg_construct); whole-array
// form = grid-stride 128-bit loads + shuffle tree + a second one-CTA kernel
// launched with programmatic dependent launch; segment form = one warp per
// segment.
#include "common.cuh"

namespace lcpp {

template <bool IS_MAX, typename T>
__device__ __forceinline__ void arg_combine(T& v, uint32_t& i, T v2, uint32_t i2) {
    const bool take = IS_MAX ? (v2 > v || (v2 == v && i2 > i)) : (v2 < v || (v2 == v && i2 < i));
    if (take) {
        v = v2;
        i = i2;
    }
}

template <bool IS_MAX, typename T>
__device__ __forceinline__ void arg_warp_reduce(T& v, uint32_t& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const T v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t i2 = __shfl_xor_sync(0xffffffffu, i, o);
        arg_combine<IS_MAX>(v, i, v2, i2);
    }
}

template <bool IS_MAX, typename T>
__device__ __forceinline__ T arg_identity() {
    return IS_MAX ? Limits<T>::lowest() : Limits<T>::max();
}

// Identity index: loses every tie against a real element.
template <bool IS_MAX>
__device__ __forceinline__ uint32_t arg_identity_index() {
    return IS_MAX ? 0u : 0xffffffffu;
}

constexpr int ARG_THREADS = 512;
constexpr int ARG_MAX_GRID = 148 * 8;

template <bool IS_MAX, typename T>
__global__ void __launch_bounds__(ARG_THREADS)
arg_partial_kernel(const T* __restrict__ in, uint64_t n, T* __restrict__ pv, uint32_t* __restrict__ pi) {
    constexpr int VEC = 16 / sizeof(T);
    __shared__ T s_v[ARG_THREADS / 32];
    __shared__ uint32_t s_i[ARG_THREADS / 32];
    T v = arg_identity<IS_MAX, T>();
    uint32_t idx = arg_identity_index<IS_MAX>();
    const uint64_t mis = (reinterpret_cast<uintptr_t>(in) & 15) / sizeof(T);
    uint64_t head = mis ? (uint64_t)(VEC - mis) : 0;
    if (head > n) head = n;
    const uint64_t gtid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t gstride = (uint64_t)gridDim.x * blockDim.x;
    if (gtid < head) arg_combine<IS_MAX>(v, idx, in[gtid], (uint32_t)gtid);
    const uint4* vin = reinterpret_cast<const uint4*>(in + head);
    const uint64_t nvec = (n - head) / VEC;
    for (uint64_t i = gtid; i < nvec; i += gstride) {
        const uint4 q = ld_stream(vin + i);
        const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
        for (int k = 0; k < VEC; ++k) arg_combine<IS_MAX>(v, idx, e[k], (uint32_t)(head + i * VEC + k));
    }
    const uint64_t t0 = head + nvec * VEC;
    if (t0 + gtid < n) arg_combine<IS_MAX>(v, idx, in[t0 + gtid], (uint32_t)(t0 + gtid));
    arg_warp_reduce<IS_MAX>(v, idx);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        s_v[warp] = v;
        s_i[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
        v = lane < ARG_THREADS / 32 ? s_v[lane] : arg_identity<IS_MAX, T>();
        idx = lane < ARG_THREADS / 32 ? s_i[lane] : arg_identity_index<IS_MAX>();
        arg_warp_reduce<IS_MAX>(v, idx);
        if (lane == 0) {
            pv[blockIdx.x] = v;
            pi[blockIdx.x] = idx;
        }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <bool IS_MAX, typename T>
__global__ void __launch_bounds__(32)
arg_final_kernel(const T* __restrict__ pv, const uint32_t* __restrict__ pi, unsigned count, uint64_t n,
                 T* __restrict__ out_v, uint32_t* __restrict__ out_i) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    T v = arg_identity<IS_MAX, T>();
    uint32_t idx = arg_identity_index<IS_MAX>();
    for (unsigned b = threadIdx.x; b < count; b += 32) arg_combine<IS_MAX>(v, idx, pv[b], pi[b]);
    arg_warp_reduce<IS_MAX>(v, idx);
    if (threadIdx.x == 0) {
        if (n == 0) idx = 1;  // empty input: {1, identity}
        *out_v = v;
        *out_i = idx;
    }
}

template <bool IS_MAX, typename T, bool FIXED>
__global__ void __launch_bounds__(256)
seg_arg_kernel(const T* __restrict__ in, T* __restrict__ out_v, uint32_t* __restrict__ out_i, uint64_t S,
               const uint32_t* __restrict__ begin, const uint32_t* __restrict__ end, uint64_t seg_size) {
    const int lane = threadIdx.x & 31;
    const uint64_t s = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (s >= S) return;
    uint64_t b, e;
    if (FIXED) {
        b = s * seg_size;
        e = b + seg_size;
    } else {
        b = __ldg(begin + s);
        e = __ldg(end + s);
        if (e < b) e = b;
    }
    T v = arg_identity<IS_MAX, T>();
    uint32_t idx = arg_identity_index<IS_MAX>();
    for (uint64_t i = b + lane; i < e; i += 32) arg_combine<IS_MAX>(v, idx, ldcs(in + i), (uint32_t)(i - b));
    arg_warp_reduce<IS_MAX>(v, idx);
    if (lane == 0) {
        out_v[s] = v;
        out_i[s] = e == b ? 1u : idx;
    }
}

template <bool IS_MAX, typename T>
static lcpp_status arg_launch(const void* in, void* out_v, uint32_t* out_i, uint64_t n, void* temp, cudaStream_t s) {
    const DeviceInfo di = device_info();
    uint64_t g = ceil_div(n ? n : 1, (uint64_t)ARG_THREADS * (16 / sizeof(T)) * 4);
    uint64_t cap = (uint64_t)di.sms * 4;
    if (cap > ARG_MAX_GRID) cap = ARG_MAX_GRID;
    if (g > cap) g = cap;
    T* pv = (T*)temp;
    uint32_t* pi = (uint32_t*)((char*)temp + align_up((size_t)ARG_MAX_GRID * sizeof(T), 256));
    arg_partial_kernel<IS_MAX, T><<<(unsigned)g, ARG_THREADS, 0, s>>>((const T*)in, n, pv, pi);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, arg_final_kernel<IS_MAX, T>, (const T*)pv, (const uint32_t*)pi, (unsigned)g, n,
                           (T*)out_v, out_i) != cudaSuccess)
        return LCPP_ERR_CUDA;
    count_launch(2);
    return check_launch();
}

}  // namespace lcpp

using namespace lcpp;

extern "C" size_t lcpp_arg_reduce_temp_bytes(int dtype, uint64_t n) {
    (void)n;
    const size_t es = lcpp_dtype_size(dtype);
    if (!es) return 0;
    return align_up((size_t)ARG_MAX_GRID * es, 256) + align_up((size_t)ARG_MAX_GRID * 4, 256);
}

extern "C" lcpp_status lcpp_arg_reduce(int op, int dtype, const void* in, void* out_value, uint32_t* out_index,
                                       uint64_t n, void* temp, size_t temp_bytes, void* stream) {
    if ((op != LCPP_OP_MIN && op != LCPP_OP_MAX) || !out_value || !out_index || (n && !in) ||
        n >= (1ull << 32))
        return LCPP_ERR_INVALID_ARG;
    const size_t need = lcpp_arg_reduce_temp_bytes(dtype, n);
    if (!need) return LCPP_ERR_INVALID_ARG;
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    cudaStream_t s = (cudaStream_t)stream;
    return dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        ProfScope ps("arg_reduce", s);
        return op == LCPP_OP_MAX ? arg_launch<true, T>(in, out_value, out_index, n, temp, s)
                                 : arg_launch<false, T>(in, out_value, out_index, n, temp, s);
    });
}

static lcpp_status seg_arg(int op, int dtype, const void* in, void* out_value, uint32_t* out_index, uint64_t S,
                           const uint32_t* begin, const uint32_t* end, uint64_t seg_size, bool fixed,
                           cudaStream_t s) {
    return dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        const unsigned g = (unsigned)ceil_div(S, 8);
        const T* pin = (const T*)in;
        T* pv = (T*)out_value;
        if (op == LCPP_OP_MAX) {
            if (fixed) seg_arg_kernel<true, T, true><<<g, 256, 0, s>>>(pin, pv, out_index, S, begin, end, seg_size);
            else seg_arg_kernel<true, T, false><<<g, 256, 0, s>>>(pin, pv, out_index, S, begin, end, seg_size);
        } else {
            if (fixed) seg_arg_kernel<false, T, true><<<g, 256, 0, s>>>(pin, pv, out_index, S, begin, end, seg_size);
            else seg_arg_kernel<false, T, false><<<g, 256, 0, s>>>(pin, pv, out_index, S, begin, end, seg_size);
        }
        count_launch();
        return check_launch();
    });
}

extern "C" lcpp_status lcpp_segment_arg_reduce(int op, int dtype, const void* in, void* out_value,
                                               uint32_t* out_index, uint64_t num_segments,
                                               const uint32_t* begin_offsets, const uint32_t* end_offsets,
                                               void* stream) {
    if ((op != LCPP_OP_MIN && op != LCPP_OP_MAX) || !lcpp_dtype_size(dtype)) return LCPP_ERR_INVALID_ARG;
    if (num_segments == 0) return LCPP_OK;
    if (!out_value || !out_index || !begin_offsets || !end_offsets || num_segments > 0xffffffffull)
        return LCPP_ERR_INVALID_ARG;
    return seg_arg(op, dtype, in, out_value, out_index, num_segments, begin_offsets, end_offsets, 0, false,
                   (cudaStream_t)stream);
}

extern "C" lcpp_status lcpp_segment_arg_reduce_fixed(int op, int dtype, const void* in, void* out_value,
                                                     uint32_t* out_index, uint64_t num_segments,
                                                     uint64_t segment_size, void* stream) {
    if ((op != LCPP_OP_MIN && op != LCPP_OP_MAX) || !lcpp_dtype_size(dtype)) return LCPP_ERR_INVALID_ARG;
    if (num_segments == 0) return LCPP_OK;
    if (!out_value || !out_index || (!in && segment_size) || segment_size >= (1ull << 32))
        return LCPP_ERR_INVALID_ARG;
    return seg_arg(op, dtype, in, out_value, out_index, num_segments, nullptr, nullptr, segment_size, true,
                   (cudaStream_t)stream);
}
