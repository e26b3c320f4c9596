/*
 * lcpp/runtime/core.h — headless runtime shim + module base for the B200
 * build of LCPP's public API.
 *
 * The reference's public classes live on LuisaCompute (Device, Stream,
 * CommandList, Buffer<T>, BufferView<T>; src/lcpp/runtime/core.h:10-112).
 * This header provides just the part of that API the Device* classes and
 * their callers use, over the CUDA runtime: a Device is a CUDA ordinal, a
 * Stream a cudaStream_t, a Buffer<T> a cudaMalloc'd array, a CommandList a
 * list of deferred commands run in order when committed to a Stream.  There is
 * no JIT (the reference's lazy_compile, core.h:36-50): kernels are compiled
 * ahead of time into liblcpp_b200.so.
 *
 * Link with -llcpp_b200 -lcudart.
 */
#pragma once

#include <cuda_runtime.h>

#include <cassert>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <string_view>
#include <type_traits>
#include <utility>
#include <vector>

#include "lcpp_b200.h"

namespace luisa {
using uint = uint32_t;
using int32 = int32_t;
using uint64 = uint64_t;
using ulong = uint64_t;
template <typename T>
using vector = std::vector<T>;
using string = std::string;
using string_view = std::string_view;
}  // namespace luisa

namespace luisa::compute {

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// One deferred step recorded into a CommandList or sent to a Stream.  It
// returns an lcpp_status (0 on success).
using Command = std::function<int(cudaStream_t)>;

template <typename T>
class BufferView {
  public:
    BufferView() = default;
    BufferView(T* ptr, size_t n) : ptr_(ptr), n_(n) {}
    T* data() const noexcept { return ptr_; }
    size_t size() const noexcept { return n_; }
    size_t size_bytes() const noexcept { return n_ * sizeof(T); }
    BufferView subview(size_t offset, size_t count) const {
        if (offset + count > n_) throw std::out_of_range("BufferView::subview");
        return BufferView(ptr_ + offset, count);
    }
    template <typename U>
    BufferView<U> as() const {
        return BufferView<U>(reinterpret_cast<U*>(ptr_), n_ * sizeof(T) / sizeof(U));
    }
    Command copy_from(const void* host) const {
        T* p = ptr_;
        const size_t b = size_bytes();
        return [p, host, b](cudaStream_t s) {
            return cudaMemcpyAsync(p, host, b, cudaMemcpyHostToDevice, s) == cudaSuccess ? 0 : LCPP_ERR_CUDA;
        };
    }
    Command copy_to(void* host) const {
        T* p = ptr_;
        const size_t b = size_bytes();
        return [p, host, b](cudaStream_t s) {
            return cudaMemcpyAsync(host, p, b, cudaMemcpyDeviceToHost, s) == cudaSuccess ? 0 : LCPP_ERR_CUDA;
        };
    }

  private:
    T* ptr_ = nullptr;
    size_t n_ = 0;
};

template <typename T>
class Buffer {
  public:
    Buffer() = default;
    explicit Buffer(size_t n) : n_(n) {
        void* p = nullptr;
        if (n) cuda_check(cudaMalloc(&p, n * sizeof(T)), "cudaMalloc");
        mem_ = std::shared_ptr<void>(p, [](void* q) { if (q) cudaFree(q); });
    }
    BufferView<T> view() const { return BufferView<T>(static_cast<T*>(mem_.get()), n_); }
    BufferView<T> view(size_t offset, size_t count) const { return view().subview(offset, count); }
    operator BufferView<T>() const { return view(); }
    size_t size() const noexcept { return n_; }
    T* data() const noexcept { return static_cast<T*>(mem_.get()); }
    Command copy_from(const void* host) const { return view().copy_from(host); }
    Command copy_to(void* host) const { return view().copy_to(host); }

  private:
    std::shared_ptr<void> mem_;
    size_t n_ = 0;
};

struct CommitCommand {
    std::vector<Command> cmds;
};
struct SynchronizeCommand {};
inline SynchronizeCommand synchronize() { return {}; }

class CommandList {
  public:
    CommandList& operator<<(Command c) {
        cmds_.push_back(std::move(c));
        return *this;
    }
    size_t size() const noexcept { return cmds_.size(); }
    bool empty() const noexcept { return cmds_.empty(); }
    CommitCommand commit() {
        CommitCommand c{std::move(cmds_)};
        cmds_.clear();
        return c;
    }

  private:
    std::vector<Command> cmds_;
};

class Stream {
  public:
    Stream() = default;
    explicit Stream(int device) : device_(device) {
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        cudaStream_t s = nullptr;
        cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
        s_ = std::shared_ptr<CUstream_st>(s, [](cudaStream_t q) { if (q) cudaStreamDestroy(q); });
    }
    cudaStream_t handle() const noexcept { return s_.get(); }
    // Status of the first failed command since the last synchronize() (0 if none).
    int last_status() const noexcept { return status_; }

    Stream& operator<<(const Command& c) {
        record(c(handle()));
        return *this;
    }
    Stream& operator<<(CommitCommand c) {
        for (auto& cmd : c.cmds) record(cmd(handle()));
        return *this;
    }
    Stream& operator<<(SynchronizeCommand) {
        cuda_check(cudaStreamSynchronize(handle()), "cudaStreamSynchronize");
        return *this;
    }
    void synchronize() { *this << compute::synchronize(); }

  private:
    void record(int st) {
        if (st != 0 && status_ == 0) status_ = st;
    }
    int device_ = 0;
    std::shared_ptr<CUstream_st> s_;
    int status_ = 0;
};

class Device {
  public:
    Device() = default;
    explicit Device(int ordinal) : ordinal_(ordinal) {}
    int ordinal() const noexcept { return ordinal_; }
    Stream create_stream() const { return Stream(ordinal_); }
    template <typename T>
    Buffer<T> create_buffer(size_t n) const {
        cuda_check(cudaSetDevice(ordinal_), "cudaSetDevice");
        return Buffer<T>(n);
    }

  private:
    int ordinal_ = 0;
};

// Only the "cuda" backend exists; the reference's DirectX/Metal/Vulkan/CPU
// backends have no counterpart.
class Context {
  public:
    Context() = default;
    explicit Context(std::string_view /*program_path*/) {}
    Device create_device(std::string_view backend = "cuda", int ordinal = 0) const {
        if (backend != "cuda") throw std::invalid_argument("only the cuda backend is available");
        return Device(ordinal);
    }
};

}  // namespace luisa::compute

namespace luisa::parallel_primitive {

namespace details {
// Tile constants of the reference (runtime/core.h:19-22).  They remain the
// class templates' default arguments; the sm_100a kernels choose their own
// tile shapes.
constexpr static size_t WARP_SIZE = 32;
constexpr static size_t BLOCK_SIZE = 256;
constexpr static size_t ITEMS_PER_THREAD = 4;
constexpr static size_t LOG_WARP_SIZE = 5;
}  // namespace details

// Element type -> lcpp_dtype.
template <typename T>
constexpr int lcpp_dtype_of() {
    if constexpr (std::is_same_v<T, int32_t>) return LCPP_I32;
    else if constexpr (std::is_same_v<T, uint32_t>) return LCPP_U32;
    else if constexpr (std::is_same_v<T, float>) return LCPP_F32;
    else if constexpr (std::is_integral_v<T> && std::is_signed_v<T> && sizeof(T) == 8) return LCPP_I64;
    else if constexpr (std::is_integral_v<T> && std::is_unsigned_v<T> && sizeof(T) == 8) return LCPP_U64;
    else if constexpr (std::is_same_v<T, double>) return LCPP_F64;
    else return -1;
}

// Reduction / scan operators of the reference (common/thread_operators.h:
// SumOp, MinOp, MaxOp).  Here they only select the kernel's operator.
struct SumOp { static constexpr int lcpp_op = LCPP_OP_SUM; };
struct MinOp { static constexpr int lcpp_op = LCPP_OP_MIN; };
struct MaxOp { static constexpr int lcpp_op = LCPP_OP_MAX; };
// Element transforms for DeviceReduce::TransformReduce (the reference's DSL
// transform lambdas cannot cross the C ABI).
struct IdentityOp { static constexpr int lcpp_xf = LCPP_XF_IDENTITY; };
struct SquareOp { static constexpr int lcpp_xf = LCPP_XF_SQUARE; };
struct AbsOp { static constexpr int lcpp_xf = LCPP_XF_ABS; };
struct NegateOp { static constexpr int lcpp_xf = LCPP_XF_NEGATE; };

template <typename T>
concept NumericT = std::is_integral_v<T> || std::is_floating_point_v<T>;

// Reference: lcpp_check (runtime/core.h:57-66) — in debug builds commit the
// list on the debug stream, synchronize and assert success; a no-op in release.
inline void lcpp_check(luisa::compute::CommandList& cmdlist, luisa::compute::Stream* debug_stream) {
#ifndef NDEBUG
    if (debug_stream) {
        *debug_stream << cmdlist.commit() << luisa::compute::synchronize();
        assert(debug_stream->last_status() == 0 && "lcpp_check failed");
    }
#else
    (void)cmdlist;
    (void)debug_stream;
#endif
}

class LuisaModule {
  protected:
    using Device = luisa::compute::Device;
    using Stream = luisa::compute::Stream;
    using CommandList = luisa::compute::CommandList;
    template <typename T>
    using Buffer = luisa::compute::Buffer<T>;
    template <typename T>
    using BufferView = luisa::compute::BufferView<T>;
    using uint = luisa::uint;
};

// Helpers of the reference's common/utils.h:49,160-169.
template <typename T>
constexpr T ceil_div(T a, T b) { return (a + b - 1) / b; }
inline size_t align_up_uint(size_t byte_offset, size_t alignment) {
    return (byte_offset + alignment - 1) / alignment * alignment;
}
inline size_t bytes_to_uint_count(size_t byte_size) { return (byte_size + sizeof(uint32_t) - 1) / sizeof(uint32_t); }

}  // namespace luisa::parallel_primitive
