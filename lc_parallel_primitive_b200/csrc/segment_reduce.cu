// DeviceSegmentReduce for sm_100a with segment-length-aware mapping.
//
// Reference behaviour followed: segment_reduce_array_recursive
// (src/lcpp/device/device_segment_reduce.h:353-381) and its kernel
// (src/lcpp/device/details/segment_reduce.h:43-86): out[s] = init (+)
// reduce(in[begin[s]..end[s])), empty segment -> init; fixed-size variant
// (details/segment_reduce.h:98-164).  The reference runs one 256-thread CTA
// per segment; at 2^20 segments of ~128 items most of those threads idle.
//
// B200 mapping:
//  * Kernel A: one warp per segment (8 segments per 256-thread CTA), lanes
//    read consecutive elements (4 independent loads in flight per lane).  A
//    segment longer than SEG_LONG is not reduced here: its id is appended to a
//    work list in temp.
//  * Kernel B: persistent CTAs (2 per SM) take long segments from that list
//    and reduce each with a whole 512-thread CTA using 128-bit loads.
// Each segment is reduced by exactly one warp or one CTA in a fixed order, so
// float results do not depend on scheduling.
#include "common.cuh"

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
                          const uint32_t* end, uint64_t seg_size, bool fixed, void* temp, cudaStream_t s) {
    switch (op) {
        case LCPP_OP_SUM: return seg_launch<OpSum, T>(in, out, S, begin, end, seg_size, fixed, temp, s);
        case LCPP_OP_MIN: return seg_launch<OpMin, T>(in, out, S, begin, end, seg_size, fixed, temp, s);
        default: return seg_launch<OpMax, T>(in, out, S, begin, end, seg_size, fixed, temp, s);
    }
}

}  // namespace lcpp

using namespace lcpp;

extern "C" size_t lcpp_segment_reduce_temp_bytes(int dtype, uint64_t num_items, uint64_t num_segments) {
    (void)num_items;
    if (!lcpp_dtype_size(dtype)) return 0;
    return SEG_HDR + align_up((num_segments ? num_segments : 1) * sizeof(uint32_t), 256);
}

extern "C" lcpp_status lcpp_segment_reduce(int op, int dtype, const void* in, void* out,
                                           uint64_t num_segments, const uint32_t* begin_offsets,
                                           const uint32_t* end_offsets, void* temp,
                                           size_t temp_bytes, void* stream) {
    if (op < 0 || op > 2 || !lcpp_dtype_size(dtype)) return LCPP_ERR_INVALID_ARG;
    if (num_segments == 0) return LCPP_OK;
    if (!out || !begin_offsets || !end_offsets || num_segments > 0xffffffffull) return LCPP_ERR_INVALID_ARG;
    // Without enough temp for the long-segment work list the call still runs:
    // one warp per segment, long ones included (slower on very long segments).
    if (!temp || temp_bytes < lcpp_segment_reduce_temp_bytes(dtype, 0, num_segments)) temp = nullptr;
    return dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        return seg_op<T>(op, in, out, num_segments, begin_offsets, end_offsets, 0, false, temp,
                         (cudaStream_t)stream);
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
