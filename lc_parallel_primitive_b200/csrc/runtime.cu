// Library-wide state: the per-device error word, the look-back wait cap,
// device attribute cache, launch counter and small ABI helpers.
#include "common.cuh"
#include <mutex>
#include <vector>

namespace lcpp {



static std::vector<UnitHook>& unit_hooks() {
    static std::vector<UnitHook> hooks;
    return hooks;
}
void register_unit_hook(UnitHook hook) { unit_hooks().push_back(hook); }

DeviceInfo device_info() {
    static std::mutex mu;
    static DeviceInfo cache[64];
    static bool have[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DeviceInfo{};
    std::lock_guard<std::mutex> g(mu);
    if (!have[dev]) {
        DeviceInfo d;
        d.device = dev;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0)
            d.sms = sms;
        cache[dev] = d;
        have[dev] = true;
    }
    return cache[dev];
}

}  // namespace lcpp

using namespace lcpp;

extern "C" const char* lcpp_status_string(lcpp_status s) {
    switch (s) {
        case LCPP_OK: return "ok";
        case LCPP_ERR_INVALID_ARG: return "invalid argument";
        case LCPP_ERR_TEMP_TOO_SMALL: return "temp storage too small";
        case LCPP_ERR_CUDA: return "CUDA error";
        case LCPP_ERR_LOOKBACK_TIMEOUT: return "look-back wait timed out";
        case LCPP_ERR_NCCL: return "NCCL error";
        case LCPP_ERR_UNSUPPORTED: return "unsupported";
        case LCPP_ERR_CAPACITY: return "output capacity exceeded";
        default: return "unknown status";
    }
}

extern "C" size_t lcpp_dtype_size(int dtype) {
    switch (dtype) {
        case LCPP_I32: case LCPP_U32: case LCPP_F32: return 4;
        case LCPP_I64: case LCPP_U64: case LCPP_F64: return 8;
        case LCPP_NONE: return 0;
        default: return 0;
    }
}

extern "C" lcpp_status lcpp_last_device_error(void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    unsigned int first = 0;
    for (UnitHook h : unit_hooks()) {  // every unit's word, each read and cleared
        unsigned int err = 0;
        if (h(0, &err, s) != 0) return LCPP_ERR_CUDA;
        if (!first) first = err;
    }
    return (lcpp_status)(int)first;
}

extern "C" lcpp_status lcpp_set_spin_limit(uint32_t iterations) {
    unsigned int v = iterations ? iterations : (1u << 22);
    for (UnitHook h : unit_hooks())
        if (h(1, &v, nullptr) != 0) return LCPP_ERR_CUDA;
    return LCPP_OK;
}

namespace lcpp {
// Compiled with the same flags as every kernel of the library.
__global__ void lcpp_arch_probe_kernel() {}
}  // namespace lcpp

extern "C" int lcpp_kernel_binary_version(void) {
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, lcpp_arch_probe_kernel) != cudaSuccess) return LCPP_ERR_CUDA;
    return a.binaryVersion;
}

extern "C" uint64_t lcpp_kernel_launch_count(void) { return g_launches.load(); }

extern "C" const char* lcpp_build_info(void) {
#define LCPP_STR2(x) #x
#define LCPP_STR(x) LCPP_STR2(x)
    return "liblcpp_b200: sm_100a, nvcc " LCPP_STR(__CUDACC_VER_MAJOR__) "." LCPP_STR(__CUDACC_VER_MINOR__);
}

extern "C" lcpp_status lcpp_profile_enable(int on) {
    Profiler& p = profiler();
    std::lock_guard<std::mutex> g(p.mu);
    for (auto& r : p.pending) { cudaEventDestroy(r.start); cudaEventDestroy(r.stop); }
    p.pending.clear();
    p.totals.clear();
    p.enabled.store(on ? 1 : 0);
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_profile_read(const char* kernel, uint64_t* launches, double* total_ms) {
    if (!kernel || !launches || !total_ms) return LCPP_ERR_INVALID_ARG;
    Profiler& p = profiler();
    std::lock_guard<std::mutex> g(p.mu);
    for (auto& r : p.pending) {
        if (cudaEventSynchronize(r.stop) != cudaSuccess) return LCPP_ERR_CUDA;
        float ms = 0;
        cudaEventElapsedTime(&ms, r.start, r.stop);
        auto& t = p.totals[r.name];
        t.first += 1;
        t.second += ms;
        cudaEventDestroy(r.start);
        cudaEventDestroy(r.stop);
    }
    p.pending.clear();
    auto it = p.totals.find(kernel);
    *launches = it == p.totals.end() ? 0 : it->second.first;
    *total_ms = it == p.totals.end() ? 0.0 : it->second.second;
    return LCPP_OK;
}
