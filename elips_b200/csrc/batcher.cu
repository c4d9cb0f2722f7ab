// Dynamic batching of single-query searches: the device counterpart of
// elips::gpu::DynamicBatcher (src/gpu_engine/DynamicBatcher.cpp:1-124,
// include/elips/gpu_engine/DynamicBatcher.hpp). Concurrent callers (Vault::seek
// readers) each submit one query; a worker thread waits up to `window_us`
// for up to `max_batch` queries, packs them into one pinned buffer, runs ONE
// fused exact search over the device index for the whole batch, and hands
// every caller its own rows. Per-query results do not depend on which other
// queries share the batch (each query's top-k is exact with ties by row), so
// they equal a direct search.
//
// Differences from the reference, both deliberate: each caller gets its own
// k (the batch is searched with the largest k and every caller takes its
// prefix; the reference passes the first query's k to the whole batch), and
// queries still pending at shutdown are served before the worker exits.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <future>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/elips_b200.h"
#include "engine.cuh"
#include "capi_util.cuh"

struct elips_b200_exact {
    eb::ExactIndex index;
};

namespace eb {
namespace {

class Batcher {
public:
    Batcher(const ExactIndex& index, size_t window_us, size_t max_batch)
        : index_(index), window_us_(window_us), max_batch_(std::max<size_t>(1, max_batch)) {
        in_elem_ = index.kind() == OperandKind::I8 ? 1 : 4;
        q_bytes_ = static_cast<size_t>(index.dim()) * in_elem_;
        DeviceGuard g(index.device());
        check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), ELIPS_B200_INITIALIZATION_FAILED,
                   "cudaStreamCreate");
        running_ = true;
        worker_ = std::thread([this] { loop(); });
    }

    ~Batcher() {
        {
            std::lock_guard<std::mutex> lock(mu_);
            running_ = false;
        }
        cv_.notify_all();
        idle_cv_.notify_all();
        if (worker_.joinable()) worker_.join();
        // Destructors must not throw: plain calls, errors ignored.
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(index_.device());
        if (host_ != nullptr) cudaFreeHost(host_);
        if (dev_ != nullptr) cudaFree(dev_);
        cudaStreamDestroy(stream_);
        if (prev >= 0) cudaSetDevice(prev);
    }

    // Blocks until this query's batch has run; returns its status.
    int search(const void* query, size_t k, float* out_dist, int64_t* out_rows) {
        Pending p;
        p.query.resize(q_bytes_);
        std::memcpy(p.query.data(), query, q_bytes_);
        p.k = k;
        p.dist = out_dist;
        p.rows = out_rows;
        std::future<int> done = p.status.get_future();
        {
            std::lock_guard<std::mutex> lock(mu_);
            if (!running_) return ELIPS_B200_BACKEND_UNAVAILABLE;
            p.ticket = enqueued_++;
            pending_.push_back(std::move(p));
            if (pending_.size() >= max_batch_) cv_.notify_one();
        }
        cv_.notify_one();
        return done.get();
    }

    // Dispatches the queries pending at the call without the window and
    // waits until the worker has served them (DynamicBatcher::flush,
    // DynamicBatcher.cpp:36-65). Queries enqueued after the call neither
    // extend the wait nor skip their window.
    void flush() {
        std::unique_lock<std::mutex> lock(mu_);
        const uint64_t target = enqueued_;  // tickets below this were pending at the call
        if (served_ >= target) return;
        flush_upto_ = std::max(flush_upto_, target);
        cv_.notify_all();
        idle_cv_.wait(lock, [&] { return served_ >= target || !running_; });
    }

    uint64_t pending() {
        std::lock_guard<std::mutex> lock(mu_);
        return pending_.size();
    }

    void stats(uint64_t* launches, uint64_t* queries) const {
        if (launches != nullptr) *launches = launches_.load();
        if (queries != nullptr) *queries = queries_.load();
    }

private:
    struct Pending {
        std::vector<uint8_t> query;
        size_t k = 0;
        float* dist = nullptr;
        int64_t* rows = nullptr;
        std::promise<int> status;
        uint64_t ticket = 0;  // arrival order
    };

    void loop() {
        for (;;) {
            std::vector<Pending> batch;
            {
                std::unique_lock<std::mutex> lock(mu_);
                cv_.wait(lock, [this] { return !pending_.empty() || !running_; });
                if (pending_.empty() && !running_) return;
                // The window opens with the first pending query; a flush skips
                // it while queries pending at the flush are still queued.
                cv_.wait_for(lock, std::chrono::microseconds(window_us_), [this] {
                    return pending_.size() >= max_batch_ || !running_ || pending_.front().ticket < flush_upto_;
                });
                const size_t take = std::min(pending_.size(), max_batch_);
                for (size_t i = 0; i < take; ++i) {
                    batch.push_back(std::move(pending_.front()));
                    pending_.pop_front();
                }
            }
            if (!batch.empty()) {
                launches_++;
                queries_ += batch.size();
                const int st = guarded([&] { run(batch); });
                for (auto& p : batch) p.status.set_value(st);
            }
            if (!batch.empty()) {
                std::lock_guard<std::mutex> lock(mu_);
                served_ = batch.back().ticket + 1;  // FIFO: every earlier ticket is served too
                idle_cv_.notify_all();
            }
        }
    }

    static size_t up256(size_t x) { return (x + 255) / 256 * 256; }

    // Layout of the host and device batch buffers: queries, distances, rows,
    // each section starting on a 256-byte boundary (the rows are int64).
    struct Layout {
        size_t dist, rows, end;
    };
    Layout layout(size_t nq, size_t k) const {
        Layout l;
        l.dist = up256(nq * q_bytes_);
        l.rows = l.dist + up256(nq * k * sizeof(float));
        l.end = l.rows + nq * k * sizeof(int64_t);
        return l;
    }

    void reserve(size_t nq, size_t k) {
        const size_t need = layout(nq, k).end;
        if (need <= cap_) return;
        if (host_ != nullptr) cudaFreeHost(host_);
        if (dev_ != nullptr) cudaFree(dev_);
        host_ = nullptr;
        dev_ = nullptr;
        check_cuda(cudaMallocHost(&host_, need), ELIPS_B200_INSUFFICIENT_MEMORY, "pinned batch buffer");
        check_cuda(cudaMalloc(&dev_, need), ELIPS_B200_INSUFFICIENT_MEMORY, "device batch buffer");
        cap_ = need;
    }

    void run(std::vector<Pending>& batch) {
        const size_t nq = batch.size();
        size_t kmax = 0;
        for (const auto& p : batch) kmax = std::max(kmax, p.k);
        if (kmax == 0) return;
        DeviceGuard g(index_.device());
        reserve(nq, kmax);
        uint8_t* h = static_cast<uint8_t*>(host_);
        uint8_t* d = static_cast<uint8_t*>(dev_);
        for (size_t i = 0; i < nq; ++i) std::memcpy(h + i * q_bytes_, batch[i].query.data(), q_bytes_);
        const Layout l = layout(nq, kmax);
        float* hd = reinterpret_cast<float*>(h + l.dist);
        int64_t* hr = reinterpret_cast<int64_t*>(h + l.rows);
        check_cuda(cudaMemcpyAsync(d, h, nq * q_bytes_, cudaMemcpyHostToDevice, stream_), ELIPS_B200_TRANSFER_FAILED,
                   "batch upload");
        index_.search_device(d, nq, kmax, nullptr, 0, reinterpret_cast<float*>(d + l.dist),
                             reinterpret_cast<int64_t*>(d + l.rows), nullptr, stream_);
        check_cuda(cudaMemcpyAsync(h + l.dist, d + l.dist, l.end - l.dist, cudaMemcpyDeviceToHost, stream_),
                   ELIPS_B200_TRANSFER_FAILED, "batch download");
        check_cuda(cudaStreamSynchronize(stream_), ELIPS_B200_KERNEL_LAUNCH_FAILED, "batched search");
        for (size_t i = 0; i < nq; ++i) {
            std::memcpy(batch[i].dist, hd + i * kmax, batch[i].k * sizeof(float));
            std::memcpy(batch[i].rows, hr + i * kmax, batch[i].k * sizeof(int64_t));
        }
    }

    const ExactIndex& index_;
    size_t window_us_, max_batch_, in_elem_ = 4, q_bytes_ = 0;
    cudaStream_t stream_ = nullptr;
    void* host_ = nullptr;
    void* dev_ = nullptr;
    size_t cap_ = 0;
    std::mutex mu_;
    std::condition_variable cv_;
    std::condition_variable idle_cv_;  // the queue drained and no batch runs
    std::deque<Pending> pending_;
    bool running_ = false;
    uint64_t enqueued_ = 0;    // tickets handed out
    uint64_t served_ = 0;      // every ticket below this has its results
    uint64_t flush_upto_ = 0;  // queued tickets below this skip the window
    std::thread worker_;
    std::atomic<uint64_t> launches_{0}, queries_{0};
};

}  // namespace
}  // namespace eb

struct elips_b200_batcher {
    eb::Batcher* b;
};

extern "C" {

int elips_b200_batcher_create(const elips_b200_exact* index, size_t window_us, size_t max_batch,
                              elips_b200_batcher** out) {
    if (index == nullptr || out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *out = nullptr;
    return eb::guarded([&] { *out = new elips_b200_batcher{new eb::Batcher(index->index, window_us, max_batch)}; });
}

int elips_b200_batcher_search(elips_b200_batcher* batcher, const void* query, size_t k, float* out_dist,
                              int64_t* out_rows) {
    if (batcher == nullptr || query == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (k > 0 && (out_dist == nullptr || out_rows == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    if (k == 0) return ELIPS_B200_OK;
    return eb::guarded([&] {
        const int st = batcher->b->search(query, k, out_dist, out_rows);
        if (st != ELIPS_B200_OK) eb::fail(st, "batched search failed");
    });
}

int elips_b200_batcher_stats(const elips_b200_batcher* batcher, uint64_t* launches, uint64_t* queries) {
    if (batcher == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    batcher->b->stats(launches, queries);
    return ELIPS_B200_OK;
}

int elips_b200_batcher_pending(const elips_b200_batcher* batcher, uint64_t* pending) {
    if (batcher == nullptr || pending == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *pending = batcher->b->pending();
    return ELIPS_B200_OK;
}

int elips_b200_batcher_flush(elips_b200_batcher* batcher) {
    if (batcher == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return eb::guarded([&] { batcher->b->flush(); });
}

int elips_b200_batcher_destroy(elips_b200_batcher* batcher) {
    if (batcher == nullptr) return ELIPS_B200_OK;
    return eb::guarded([&] {
        delete batcher->b;
        delete batcher;
    });
}

}  // extern "C"
