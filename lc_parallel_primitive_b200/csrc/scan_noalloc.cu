// DeviceScan without caller-provided temp storage.
//
// Some callers cannot allocate device memory at the point where they need a
// prefix sum: code running inside a custom allocator or memory-pool callback
// (where calling back into cudaMalloc would recurse or deadlock), plug-ins
// handed only pre-allocated input/output buffers by their host application,
// and real-time paths that forbid allocation after start-up.  For them this
// file keeps the scan's scratch (ticket counter + one 64-bit look-back
// descriptor per tile) in a fixed file-scope device array, so the
// call needs nothing but the input and output buffers.
//
// Limits and rules:
//  * The array holds SCAN_NOALLOC_MAX_TILES descriptors: n <= 2^29 items
//    (2 GiB of 4-byte data); larger n is rejected with
//    LCPP_ERR_INVALID_ARG.  Every GPU that loads the library holds the
//    array (~128 KiB) until the process exits.
//  * All calls on a device share the array.  Each call clears the part it
//    uses before its kernel runs, but two calls that overlap on the GPU
//    (different streams, no ordering between them) race on it: serialize
//    them.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current); make that first call
//    before any stream capture.
#include "common.cuh"
#include <mutex>
#include <vector>

namespace lcpp {

constexpr uint64_t SCAN_NOALLOC_MAX_TILES = (1ull << 29) / SCAN_TILE;  // n <= 2^29
constexpr size_t SCAN_NOALLOC_BYTES = SCAN_HDR + SCAN_NOALLOC_MAX_TILES * sizeof(uint64_t);

static __device__ __align__(256) unsigned char g_scan_noalloc_scratch[SCAN_NOALLOC_BYTES];

// Device address of g_scan_noalloc_scratch for `dev` (looked up once per
// device ordinal; the table is sized by cudaGetDeviceCount).  The cache
// assumes the device is not reset (cudaDeviceReset) while the library is
// loaded.  A first lookup while `stream` is being captured into a graph
// returns LCPP_ERR_UNSUPPORTED: make the first call on each device outside
// capture.
static lcpp_status scan_noalloc_scratch(int dev, cudaStream_t stream, void** out) {
    static std::mutex mu;
    static std::vector<void*> addr;
    std::lock_guard<std::mutex> g(mu);
    if (addr.empty()) {
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) return LCPP_ERR_CUDA;
        addr.assign((size_t)count, nullptr);
    }
    if (dev < 0 || (size_t)dev >= addr.size()) return LCPP_ERR_INVALID_ARG;
    if (!addr[dev]) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return LCPP_ERR_CUDA;
        if (cs != cudaStreamCaptureStatusNone) return LCPP_ERR_UNSUPPORTED;
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_scan_noalloc_scratch) != cudaSuccess || !p) return LCPP_ERR_CUDA;
        addr[dev] = p;
    }
    *out = addr[dev];
    return LCPP_OK;
}

}  // namespace lcpp

using namespace lcpp;

extern "C" uint64_t lcpp_scan_noalloc_max_items(void) { return SCAN_NOALLOC_MAX_TILES * SCAN_TILE; }

extern "C" lcpp_status lcpp_scan_noalloc(int kind, int dtype, const void* in, void* out, uint64_t n,
                                         void* stream) {
    if ((kind != LCPP_SCAN_EXCLUSIVE && kind != LCPP_SCAN_INCLUSIVE) || (n && (!in || !out)))
        return LCPP_ERR_INVALID_ARG;
    if (dtype != LCPP_I32 && dtype != LCPP_U32 && dtype != LCPP_F32) return LCPP_ERR_INVALID_ARG;
    if (n > SCAN_NOALLOC_MAX_TILES * SCAN_TILE) return LCPP_ERR_INVALID_ARG;  // beyond the fixed scratch
    if (n == 0) return LCPP_OK;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LCPP_ERR_CUDA;
    void* scratch = nullptr;
    const lcpp_status st = scan_noalloc_scratch(dev, (cudaStream_t)stream, &scratch);
    if (st != LCPP_OK) return st;
    const uint64_t tiles = ceil_div(n, SCAN_TILE);
    cudaStream_t s = (cudaStream_t)stream;
    unsigned int* ticket = (unsigned int*)scratch;
    uint64_t* desc = (uint64_t*)((char*)scratch + SCAN_HDR);
    // ticket and descriptors must start at zero; the array keeps the last call's contents
    if (cudaMemsetAsync(scratch, 0, SCAN_HDR + tiles * sizeof(uint64_t), s) != cudaSuccess) return LCPP_ERR_CUDA;
    auto go = [&](auto zero) -> lcpp_status {
        using T = decltype(zero);
        if (kind == LCPP_SCAN_INCLUSIVE)
            scan_kernel<OpSum, T, true><<<(unsigned)tiles, SCAN_THREADS, 0, s>>>((const T*)in, (T*)out, n, nullptr, T(0), ticket, ScanDesc<T>{desc});
        else
            scan_kernel<OpSum, T, false><<<(unsigned)tiles, SCAN_THREADS, 0, s>>>((const T*)in, (T*)out, n, nullptr, T(0), ticket, ScanDesc<T>{desc});
        count_launch();
        return check_launch();
    };
    switch (dtype) {
        case LCPP_I32: return go((int32_t)0);
        case LCPP_U32: return go((uint32_t)0);
        default: return go((float)0);
    }
}
