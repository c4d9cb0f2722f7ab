// Host-side engine: device contexts, device buffers, and the exact index.
// Everything here is C++; the C ABI in capi.cu wraps it and turns exceptions
// into status codes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "exact_topk.cuh"

namespace eb {

// Error carried from the engine to the C ABI. `code` is an ELIPS_B200_* value.
struct Error {
    int code;
    std::string what;
};

[[noreturn]] void fail(int code, const std::string& what);
void check_cuda(cudaError_t e, int code, const char* what);

// Makes `device` current for the lifetime of the guard.
class DeviceGuard {
public:
    explicit DeviceGuard(int device);
    ~DeviceGuard();
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int prev_ = -1;
};

struct DeviceProps {
    int num_sms = 0;
    int cc_major = 0, cc_minor = 0;
    size_t max_smem_optin = 0;
};

// Validates the device (sm_100), returns its properties; initialises the
// stream-ordered memory pool on first use.
const DeviceProps& device_props(int device);

// Lets `func` launch with up to `bytes` of dynamic shared memory on the
// current device. The limit is a process-wide attribute of the function, so
// it is only ever raised (under a lock): concurrent callers asking for
// different sizes never lower it below another caller's launch.
void allow_dynamic_smem(const void* func, size_t bytes);

// Owning device allocation (cudaMalloc / cudaFree).
class DeviceBuffer {
public:
    DeviceBuffer() = default;
    DeviceBuffer(int device, size_t bytes);
    ~DeviceBuffer();
    DeviceBuffer(DeviceBuffer&& o) noexcept { *this = std::move(o); }
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    void* get() const { return ptr_; }
    size_t bytes() const { return bytes_; }

private:
    void reset();
    int device_ = -1;
    void* ptr_ = nullptr;
    size_t bytes_ = 0;
};

// Stream-ordered scratch (cudaMallocAsync / cudaFreeAsync on `stream`).
class StreamScratch {
public:
    StreamScratch(size_t bytes, cudaStream_t stream);
    ~StreamScratch();
    StreamScratch(const StreamScratch&) = delete;
    StreamScratch& operator=(const StreamScratch&) = delete;
    uint8_t* get() const { return static_cast<uint8_t*>(ptr_); }

private:
    void* ptr_ = nullptr;
    cudaStream_t stream_;
};

// Builds a 2-D tiled TMA descriptor over a row-major [rows x cols] matrix
// with 128-byte swizzle and a {128 bytes, box_rows} box.
CUtensorMap make_operand_map(const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                             uint64_t cols, uint64_t rows, uint32_t box_rows);

// Partitioning of one exact search launch over `groups` MMA groups of `cg`
// CTAs (1: single CTAs, 2: CTA pairs sharing each M = 256 MMA). grid counts
// CTAs; n_qt counts query tiles of 128 * cg queries.
struct ExactPlan {
    uint32_t n_qt = 0, n_bt = 0, splits = 0, grid = 0, cap = 0, bn = 0, cg = 1;
};
ExactPlan plan_exact(uint32_t nq, uint32_t n, uint32_t k, uint32_t bn, int groups, uint32_t cg = 1);

// Device-resident brute-force index over one base shard.
class ExactIndex {
public:
    ExactIndex(int device, int metric, int precision, uint32_t dim);

    void add(const void* rows_host, size_t n);
    // rows: device memory, same element type as add(); converted on `stream`.
    void add_device(const void* rows, size_t n, cudaStream_t stream);
    // Rows ever added (the row-number space searches report in).
    size_t size() const { return n_; }
    // Rows not removed.
    size_t live() const { return n_ - removed_; }

    // Removes one row in place: its row number stays reserved and no search
    // reports it again (a tombstone bit folded into the eligibility mask), so
    // no buffer is rebuilt and the other rows keep their numbers and order.
    // Returns false when the row was already removed.
    bool remove(size_t row);
    // Drops the removed rows, keeping the others in order; new_to_old (host,
    // live() entries) receives each kept row's former number.
    void compact(uint32_t* new_to_old);

    // Device snapshot: the stored operand rows (with their norms and the
    // removal bits) as one host blob that import_blob restores into an empty
    // index of the same metric, precision and dimension without converting
    // the rows again.
    size_t blob_bytes() const;
    // Device memory this index holds: operand rows at capacity (both 3xTF32
    // planes), norms, removal bits.
    size_t device_bytes() const;
    void export_blob(void* out, size_t bytes) const;
    void import_blob(const void* blob, size_t bytes);
    int device() const { return device_; }
    int metric() const { return metric_; }
    uint32_t dim() const { return dim_; }
    OperandKind kind() const { return kind_; }

    // queries: device, nq x dim (fp32, int8 for INT8). Exactly one of
    // (out_dist, out_rows) or out_cand is used.
    // shared_bound (optional, DEVICE, may be another GPU's memory): nq
    // per-query admission bounds (ordered keys, all ones = none) shared by
    // every shard searching the same queries; the kernel reads and tightens
    // them (atomicMin) instead of private ones. The caller initialises them.
    void search_device(const void* queries, size_t nq, size_t k, const uint32_t* mask,
                       uint32_t row_offset, float* out_dist, int64_t* out_rows, uint2* out_cand,
                       cudaStream_t stream, uint32_t* shared_bound = nullptr) const;

    // The same search with all scratch carved from a caller-provided device
    // buffer of `scratch_bytes` and at most `max_grid` CTAs; performs no
    // device allocation. Fails with INVALID_ARGUMENT when the call needs more
    // scratch than the buffer holds.
    // Rows one search scans: the index's own storage, or a gathered subset.
    struct RowView {
        const void* ops;
        const void* ops_lo;
        const float* norms;
        const uint32_t* live;
        uint32_t n;
    };

    void search_device_in_scratch(const void* queries, size_t nq, size_t k, const uint32_t* mask,
                                  float* out_dist, int64_t* out_rows, uint8_t* scratch,
                                  size_t scratch_bytes, uint32_t max_grid, cudaStream_t stream) const;

private:
    void reserve(size_t rows);
    void search_rows(const RowView& rv, const void* queries, size_t nq, size_t k, const uint32_t* mask,
                     uint32_t row_offset, float* out_dist, int64_t* out_rows, uint2* out_cand,
                     cudaStream_t stream, uint32_t* shared_bound) const;
    // A row filter that selects at most half of the rows: gathers them and
    // searches the subset; false (nothing launched beyond the count) otherwise.
    bool search_gathered(const void* queries, size_t nq, size_t k, const uint32_t* mask, uint32_t row_offset,
                         float* out_dist, int64_t* out_rows, uint2* out_cand, cudaStream_t stream,
                         uint32_t* shared_bound) const;

    int device_;
    int metric_;
    int precision_;
    OperandKind kind_;
    uint32_t dim_, d_pad_, elem_bytes_;
    size_t n_ = 0, capacity_ = 0;
    DeviceBuffer ops_, ops_lo_, norms_;
    // Removal bits: created at the first remove (null = every row live).
    DeviceBuffer live_;
    std::vector<uint32_t> live_host_;
    size_t removed_ = 0;
    void mark_live(size_t first, size_t count);
    void upload_live_words(size_t w0, size_t w1);
};

// Final merge over candidate lists (see merge_topk_kernel). With sub > 1,
// the first stage of a two-stage merge: each query's lists in `sub` groups of
// `lists` (the last: lists_last), output row q*sub + j per group.
// The k (<= 256) smallest (value, index) of each of nq rows of nb distances,
// one warp per row; same results as the block top-k (values +inf and NaN
// never taken, ties by index). DEVICE pointers on `stream`.
void top_k_rows_warp(int device, const float* dist, uint32_t* idx, float* val, size_t nq, size_t nb, size_t k,
                     cudaStream_t stream);

// len: entries per candidate list (0 = k).
void merge_candidates(int device, const uint2* cand, uint32_t nq, uint32_t lists, uint32_t k,
                      uint64_t stride_q, uint64_t stride_l, int metric, float* out_dist,
                      int64_t* out_rows, uint2* out_cand, cudaStream_t stream, uint32_t sub = 1,
                      uint32_t lists_last = 0, uint32_t len = 0);

int read_and_clear_device_error(int device);
// Launches a bounded wait that must expire after `budget` cycles and returns
// the device error word it leaves (cleared again).
int wait_selftest(int device, long long budget);

}  // namespace eb
