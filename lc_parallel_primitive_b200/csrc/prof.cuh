// Optional per-kernel timing with CUDA events recorded on the launching
// stream (off by default; used by the benchmark to time the dominant kernel
// inside a full primitive call).  When disabled a scope costs one relaxed
// atomic load.
#pragma once
#include <cuda_runtime.h>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace lcpp {

struct ProfRecord {
    std::string name;
    cudaEvent_t start, stop;
};

struct Profiler {
    std::atomic<int> enabled{0};
    std::mutex mu;
    std::vector<ProfRecord> pending;
    std::unordered_map<std::string, std::pair<uint64_t, double>> totals;  // count, ms
};

inline Profiler& profiler() {
    static Profiler p;
    return p;
}

class ProfScope {
  public:
    ProfScope(const char* name, cudaStream_t s) : s_(s) {
        if (!profiler().enabled.load(std::memory_order_relaxed)) return;
        rec_.name = name;
        if (cudaEventCreate(&rec_.start) != cudaSuccess) return;
        if (cudaEventCreate(&rec_.stop) != cudaSuccess) { cudaEventDestroy(rec_.start); return; }
        cudaEventRecord(rec_.start, s_);
        on_ = true;
    }
    ~ProfScope() {
        if (!on_) return;
        cudaEventRecord(rec_.stop, s_);
        std::lock_guard<std::mutex> g(profiler().mu);
        profiler().pending.push_back(rec_);
    }

  private:
    cudaStream_t s_;
    ProfRecord rec_{};
    bool on_ = false;
};

}  // namespace lcpp
