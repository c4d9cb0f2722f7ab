// Per-kernel launch counting (always on) and CUDA-event timing (when
// enabled), the device-side counterpart of the reference's GpuProfiler
// (src/gpu_engine/GpuProfiler.cpp:5-23, record(kernel, duration, items)).
// Timing events are recorded on the launching stream around each launch and
// folded into per-kernel totals when the stats are read.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace eb {

struct KernelStats {
    uint64_t launches = 0;   // launches timed (profiling enabled)
    double total_ms = 0.0;   // summed event durations
    uint64_t items = 0;      // summed work items (e.g. query x row pairs)
};

class Profiler {
public:
    static Profiler& get() {
        static Profiler p;
        return p;
    }

    bool enabled() const { return enabled_.load(std::memory_order_relaxed); }
    void set_enabled(bool on) { enabled_.store(on, std::memory_order_relaxed); }
    uint64_t total_launches() const { return launches_.load(std::memory_order_relaxed); }

    // Brackets one kernel launch on `stream`.
    class Scope {
    public:
        Scope(const char* name, cudaStream_t stream, uint64_t items) : name_(name), stream_(stream), items_(items) {
            Profiler::get().launches_.fetch_add(1, std::memory_order_relaxed);
            if (Profiler::get().enabled() && cudaEventCreate(&start_) == cudaSuccess) {
                if (cudaEventCreate(&stop_) != cudaSuccess) {
                    cudaEventDestroy(start_);
                    start_ = nullptr;
                } else {
                    cudaEventRecord(start_, stream_);
                }
            }
        }
        ~Scope() {
            if (start_ == nullptr) return;
            cudaEventRecord(stop_, stream_);
            Profiler::get().push(name_, start_, stop_, items_);
        }
        Scope(const Scope&) = delete;
        Scope& operator=(const Scope&) = delete;

    private:
        const char* name_;
        cudaStream_t stream_;
        uint64_t items_;
        cudaEvent_t start_ = nullptr, stop_ = nullptr;
    };

    // Waits for pending events and folds them into the totals.
    void collect() {
        std::vector<Pending> pending;
        {
            std::lock_guard<std::mutex> lock(mu_);
            pending.swap(pending_);
        }
        std::map<std::string, KernelStats> add;
        for (auto& p : pending) {
            float ms = 0.0f;
            if (cudaEventSynchronize(p.stop) == cudaSuccess &&
                cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess) {
                KernelStats& s = add[p.name];
                s.launches += 1;
                s.total_ms += ms;
                s.items += p.items;
            }
            cudaEventDestroy(p.start);
            cudaEventDestroy(p.stop);
        }
        std::lock_guard<std::mutex> lock(mu_);
        for (auto& [name, s] : add) {
            KernelStats& t = totals_[name];
            t.launches += s.launches;
            t.total_ms += s.total_ms;
            t.items += s.items;
        }
    }

    // name == nullptr: sum over every kernel.
    KernelStats query(const char* name) {
        collect();
        std::lock_guard<std::mutex> lock(mu_);
        KernelStats out;
        for (auto& [n, s] : totals_) {
            if (name != nullptr && n != name) continue;
            out.launches += s.launches;
            out.total_ms += s.total_ms;
            out.items += s.items;
        }
        return out;
    }

    void reset() {
        collect();
        std::lock_guard<std::mutex> lock(mu_);
        totals_.clear();
    }

private:
    struct Pending {
        std::string name;
        cudaEvent_t start, stop;
        uint64_t items;
    };
    void push(const char* name, cudaEvent_t a, cudaEvent_t b, uint64_t items) {
        std::lock_guard<std::mutex> lock(mu_);
        pending_.push_back({name, a, b, items});
    }

    std::atomic<bool> enabled_{false};
    std::atomic<uint64_t> launches_{0};
    std::mutex mu_;
    std::vector<Pending> pending_;
    std::map<std::string, KernelStats> totals_;
};

}  // namespace eb
