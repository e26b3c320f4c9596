// Shared device/host helpers for the sm_100a primitives.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <atomic>
#include <string.h>
#include "lcpp_b200.h"
#include "prof.cuh"

namespace lcpp {

constexpr int WARP = 32;

// ---------------------------------------------------------------------------
// Device-side error word and look-back wait cap (one per device, per process).
// ---------------------------------------------------------------------------
// The library is built from a few compilation units (whole-program device
// code in each, no relocatable device code, which slowed the short two-kernel
// reduce by 16 us).  Each unit has its own copy of these words; every unit
// registers a host hook, and lcpp_last_device_error / lcpp_set_spin_limit
// walk all of them.
static __device__ unsigned int g_error = 0;               // first latched lcpp_status (as unsigned)
static __device__ unsigned int g_spin_limit = 1u << 22;   // polls before a wait gives up (~1 s)

// op 0: read this unit's error word into *value and clear it (async on s);
// op 1: set this unit's spin limit to *value.
using UnitHook = int (*)(int op, unsigned int* value, cudaStream_t s);
void register_unit_hook(UnitHook hook);  // runtime.cu
static int unit_words_hook(int op, unsigned int* value, cudaStream_t s) {
    if (op == 0) {
        const unsigned int zero = 0;
        if (cudaMemcpyFromSymbolAsync(value, g_error, sizeof(unsigned int), 0, cudaMemcpyDeviceToHost, s) !=
                cudaSuccess ||
            cudaMemcpyToSymbolAsync(g_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess)
            return -1;
        return 0;
    }
    return cudaMemcpyToSymbol(g_spin_limit, value, sizeof(unsigned int)) == cudaSuccess ? 0 : -1;
}
static const int unit_words_registered = (register_unit_hook(unit_words_hook), 0);

__device__ __forceinline__ void set_error(int status) {
    atomicCAS(&g_error, 0u, (unsigned int)status);
}

// Number of kernels launched by this library (host counter, all devices).
inline std::atomic<uint64_t> g_launches{0};
inline void count_launch(uint64_t k = 1) { g_launches.fetch_add(k, std::memory_order_relaxed); }

// ---------------------------------------------------------------------------
// Relaxed device-scope loads/stores for look-back descriptors.  Value and
// status travel in one aligned word, so no further ordering is needed.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Streaming (read-once) vector load that does not allocate in L1.
template <typename V>
__device__ __forceinline__ V ld_stream(const V* p) { return __ldcs(p); }

// Streaming scalar load/store of any 4- or 8-byte trivially copyable type.
template <typename T>
__device__ __forceinline__ T ldcs(const T* p) {
    static_assert(sizeof(T) == 4 || sizeof(T) == 8, "4- or 8-byte element");
    T r;
    if constexpr (sizeof(T) == 4) {
        const unsigned int v = __ldcs(reinterpret_cast<const unsigned int*>(p));
        memcpy(&r, &v, 4);
    } else {
        const unsigned long long v = __ldcs(reinterpret_cast<const unsigned long long*>(p));
        memcpy(&r, &v, 8);
    }
    return r;
}
template <typename T>
__device__ __forceinline__ void stcs(T* p, T x) {
    static_assert(sizeof(T) == 4 || sizeof(T) == 8, "4- or 8-byte element");
    if constexpr (sizeof(T) == 4) {
        unsigned int v;
        memcpy(&v, &x, 4);
        __stcs(reinterpret_cast<unsigned int*>(p), v);
    } else {
        unsigned long long v;
        memcpy(&v, &x, 8);
        __stcs(reinterpret_cast<unsigned long long*>(p), v);
    }
}

// 16-byte global -> shared asynchronous copy (cp.async, L2 only) and its group waits.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_prior1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// ---------------------------------------------------------------------------
// Operators.  Integer sums wrap: they are done on the unsigned bit type.
// ---------------------------------------------------------------------------
template <typename T> struct Unsigned { using type = T; };
template <> struct Unsigned<int32_t> { using type = uint32_t; };
template <> struct Unsigned<int64_t> { using type = uint64_t; };

template <typename T> struct Limits;
template <> struct Limits<int32_t>  { static __host__ __device__ int32_t  lowest() { return INT32_MIN; }  static __host__ __device__ int32_t  max() { return INT32_MAX; } };
template <> struct Limits<uint32_t> { static __host__ __device__ uint32_t lowest() { return 0u; }         static __host__ __device__ uint32_t max() { return 0xffffffffu; } };
template <> struct Limits<int64_t>  { static __host__ __device__ int64_t  lowest() { return INT64_MIN; }  static __host__ __device__ int64_t  max() { return INT64_MAX; } };
template <> struct Limits<uint64_t> { static __host__ __device__ uint64_t lowest() { return 0ull; }       static __host__ __device__ uint64_t max() { return ~0ull; } };
template <> struct Limits<float>    { static __host__ __device__ float    lowest() { return -3.40282347e+38f; } static __host__ __device__ float max() { return 3.40282347e+38f; } };
template <> struct Limits<double>   { static __host__ __device__ double   lowest() { return -1.7976931348623157e308; } static __host__ __device__ double max() { return 1.7976931348623157e308; } };

struct OpSum {
    template <typename T> static __host__ __device__ __forceinline__ T identity() { return T(0); }
    template <typename T> static __device__ __forceinline__ T apply(T a, T b) {
        using U = typename Unsigned<T>::type;
        return (T)((U)a + (U)b);
    }
};
template <> __device__ __forceinline__ float  OpSum::apply<float>(float a, float b) { return a + b; }
template <> __device__ __forceinline__ double OpSum::apply<double>(double a, double b) { return a + b; }

// Min/Max follow the reference's MinOp/MaxOp (thread_operators.h): plain
// comparisons, so a NaN operand is dropped or kept by operand position
// exactly like `a < b ? a : b`.
struct OpMin {
    template <typename T> static __host__ __device__ __forceinline__ T identity() { return Limits<T>::max(); }
    template <typename T> static __device__ __forceinline__ T apply(T a, T b) { return b < a ? b : a; }
};
struct OpMax {
    template <typename T> static __host__ __device__ __forceinline__ T identity() { return Limits<T>::lowest(); }
    template <typename T> static __device__ __forceinline__ T apply(T a, T b) { return a < b ? b : a; }
};

template <typename Op, typename T>
__device__ __forceinline__ T warp_reduce(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = Op::template apply<T>(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------
// Host helpers
// ---------------------------------------------------------------------------
struct DeviceInfo {
    int sms = 148;
    int device = 0;
};
DeviceInfo device_info();  // for the current device; cached

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

inline lcpp_status check_launch() {
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

// Dispatch a functor over the six element types.
template <typename F>
inline lcpp_status dispatch_dtype(int dtype, F&& f) {
    switch (dtype) {
        case LCPP_I32: return f((int32_t)0);
        case LCPP_U32: return f((uint32_t)0);
        case LCPP_F32: return f((float)0);
        case LCPP_I64: return f((int64_t)0);
        case LCPP_U64: return f((uint64_t)0);
        case LCPP_F64: return f((double)0);
        default: return LCPP_ERR_INVALID_ARG;
    }
}

}  // namespace lcpp
