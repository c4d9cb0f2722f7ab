// Device-resident ELIPS indexes on the B200 library: the index plugin half of
// the drop-in boundary.
//
// ELIPS selects its GPU indexes in make_index (src/IndexFactory.cpp:40-50) and
// make_gpu_index (src/gpu_engine/GpuHybridIndex.cpp:14-39); both hand back a
// GpuIndexPort (include/elips/gpu_engine/GpuIndexPort.hpp:20-45), which is an
// IndexPort (include/elips/index_engine/IndexPort.hpp:16-46) plus
// IndexTransferPort. The reference's own GpuBruteForceIndex / GpuIVFPQIndex
// reach the GPU only through GpuPort::compute_distances_batch + top_k, which
// materialise the whole query x base distance matrix on the host
// (GpuSearchPipeline.cpp:10-41). The classes here keep their rows on the
// device and search with the library's fused kernels instead:
//
//  * B200BruteForceIndex  -- GpuBruteForceIndex (GpuBruteForceIndex.cpp:77-250):
//    the fused tcgen05 distance GEMM + top-k (fp32 as 3xTF32, fp16, bf16);
//  * B200QuantizedIndex   -- ExactIndex with a Quantizer (ExactIndex.cpp:55-87,
//    sq8 / PQ / OPQ codes scanned on the device, bit-identical);
//  * B200IvfPqIndex       -- GpuIVFPQIndex (GpuIVFPQIndex.cpp:88-348) with
//    IvfIndexState's lifecycle (IvfIndexState.cpp:118-393): the model is built
//    on the device bit-identically, search is the library's probe + scan +
//    rerank.
//
// make_b200_index / make_b200_gpu_index are the two selection functions with
// these classes in place of the reference's.
//
// Semantics kept from the reference classes: type_name() strings (they start
// with "gpu_", so QueryPlan.gpu_index reports them, Database.cpp:1136);
// DimensionMismatch thrown by insert / search on a bad width; search returning
// {} when the backend fails (GpuBruteForceIndex.cpp:112,117); search_batch
// returning GpuError values; remove of an unknown id is a no-op; snapshots in
// IndexSnapshot's canonical form, so a CPU ExactIndex and these indexes
// clone into each other through GpuIndexTransferManager.
//
// GpuPrecision gains BF16 appended after Auto (GpuConfig.hpp:34: FP32, FP16,
// Int8, Auto, then BF16 = 4, nothing renumbered); until the header carries it,
// kGpuPrecisionBF16 names that value. The device a GpuConfig selects is
// config.device_index (-1 = device 0).
//
// Build: -std=c++23 -DELIPS_GPU_ENABLED -I<elips>/include -I<elips>/src/gpu_engine
// -I<this repo>/include; link libelips_b200.so.
#pragma once

#include <cstdint>
#include <memory>
#include <span>
#include <string>
#include <unordered_map>
#include <vector>

#include "elips/Config.hpp"
#include "elips/domain/RecordID.hpp"
#include "elips/gpu_engine/GpuConfig.hpp"
#include "elips/gpu_engine/GpuIndexPort.hpp"
#include "elips/index_engine/IndexPort.hpp"
#include "elips/index_engine/IndexSnapshot.hpp"
#include "elips/index_engine/IndexTransferPort.hpp"
#include "elips/quant_engine/Quantizer.hpp"

struct elips_b200_exact;
struct elips_b200_quant;
struct elips_b200_ivfpq;

namespace elips::gpu::b200 {

// GpuPrecision::BF16, appended after Auto.
inline constexpr GpuPrecision kGpuPrecisionBF16 = static_cast<GpuPrecision>(4);

class B200BruteForceIndex final : public GpuIndexPort {
public:
    B200BruteForceIndex(elips::Metric metric, std::uint16_t dimension, const GpuConfig& config);
    ~B200BruteForceIndex() override;

    void insert(const RecordID& id, std::span<const float> vector) override;
    void remove(const RecordID& id) override;
    [[nodiscard]] std::vector<Hit> search(std::span<const float> query, std::size_t k) const override;
    [[nodiscard]] std::size_t size() const noexcept override { return live_; }
    [[nodiscard]] std::string_view type_name() const noexcept override { return "gpu_brute_force"; }

    [[nodiscard]] std::expected<void, GpuError> build_from_batch(std::span<const float> vectors,
                                                                 std::span<const RecordID> ids,
                                                                 const GpuIndexBuildParams& params) override;
    [[nodiscard]] std::expected<std::vector<std::vector<SearchResult>>, GpuError>
    search_batch(std::span<const float> queries, size_t k, size_t ef_search) const override;
    // Filtered search (Vault::search_records with a candidate set,
    // Database.cpp:1065-1126): only rows whose id is in `candidates` compete.
    [[nodiscard]] std::expected<std::vector<std::vector<SearchResult>>, GpuError>
    search_batch_filtered(std::span<const float> queries, size_t k, std::span<const RecordID> candidates) const;
    [[nodiscard]] std::expected<void, GpuError> export_to_cpu_index(elips::IndexPort& cpu_index_out) const override;
    [[nodiscard]] std::expected<void, GpuError> import_from_cpu_index(const elips::IndexPort& cpu_index) override;
    [[nodiscard]] size_t device_bytes_used() const noexcept override;
    [[nodiscard]] std::string_view backend_name() const noexcept override { return "cuda"; }

    [[nodiscard]] std::expected<elips::IndexSnapshot, std::string> export_snapshot() const override;
    [[nodiscard]] std::expected<void, std::string> import_snapshot(const elips::IndexSnapshot& snapshot) override;

private:
    void reset_device();
    void compact_if_sparse();
    int search_slots(std::span<const float> queries, size_t nq, size_t k, const uint32_t* mask,
                     std::vector<float>& dist, std::vector<std::int64_t>& slots) const;
    std::expected<std::vector<std::vector<SearchResult>>, GpuError>
    search_masked(std::span<const float> queries, size_t k, const std::vector<uint32_t>* mask) const;

    elips::Metric metric_;
    std::uint16_t dimension_;
    int device_;
    int precision_;
    elips_b200_exact* h_ = nullptr;
    // slot -> id; removed slots keep their place (and their vector) until a
    // compaction, so the survivors keep the reference's relative order.
    std::vector<RecordID> slot_ids_;
    std::vector<std::uint8_t> slot_live_;
    std::vector<float> host_vectors_;  // the snapshot's fp32 source of truth, by slot
    size_t live_ = 0;
};

class B200QuantizedIndex final : public elips::IndexPort, public elips::IndexTransferPort {
public:
    B200QuantizedIndex(elips::Metric metric, std::uint16_t dimension, quant::QuantizerPtr quantizer, int device = 0);
    ~B200QuantizedIndex() override;

    void insert(const RecordID& id, std::span<const float> vector) override;
    void remove(const RecordID& id) override;
    [[nodiscard]] std::vector<Hit> search(std::span<const float> query, std::size_t k) const override;
    [[nodiscard]] std::size_t size() const noexcept override { return ids_.size(); }
    [[nodiscard]] std::string_view type_name() const noexcept override { return "gpu_exact_quantized"; }

    [[nodiscard]] std::expected<elips::IndexSnapshot, std::string> export_snapshot() const override;
    [[nodiscard]] std::expected<void, std::string> import_snapshot(const elips::IndexSnapshot& snapshot) override;

private:
    void rebuild_device();

    elips::Metric metric_;
    std::uint16_t dimension_;
    quant::QuantizerPtr quantizer_;
    int device_;
    int codec_ = 0;
    std::uint32_t pq_dim_ = 0, pq_bits_ = 0;
    std::vector<float> params_, rotation_;
    elips_b200_quant* h_ = nullptr;
    std::vector<RecordID> ids_;
    std::vector<std::uint8_t> codes_;  // host copy, row-major (ExactIndex's codes_)
};

class B200IvfPqIndex final : public GpuIndexPort {
public:
    B200IvfPqIndex(elips::Metric metric, std::uint16_t dimension, const GpuConfig& config);
    ~B200IvfPqIndex() override;

    void insert(const RecordID& id, std::span<const float> vector) override;
    void remove(const RecordID& id) override;
    [[nodiscard]] std::vector<Hit> search(std::span<const float> query, std::size_t k) const override;
    [[nodiscard]] std::size_t size() const noexcept override { return ids_.size(); }
    [[nodiscard]] std::string_view type_name() const noexcept override { return "gpu_ivf_pq"; }

    [[nodiscard]] std::expected<void, GpuError> build_from_batch(std::span<const float> vectors,
                                                                 std::span<const RecordID> ids,
                                                                 const GpuIndexBuildParams& params) override;
    [[nodiscard]] std::expected<std::vector<std::vector<SearchResult>>, GpuError>
    search_batch(std::span<const float> queries, size_t k, size_t ef_search) const override;
    [[nodiscard]] std::expected<void, GpuError> export_to_cpu_index(elips::IndexPort& cpu_index_out) const override;
    [[nodiscard]] std::expected<void, GpuError> import_from_cpu_index(const elips::IndexPort& cpu_index) override;
    [[nodiscard]] size_t device_bytes_used() const noexcept override;
    [[nodiscard]] std::string_view backend_name() const noexcept override { return "cuda"; }

    [[nodiscard]] std::expected<elips::IndexSnapshot, std::string> export_snapshot() const override;
    [[nodiscard]] std::expected<void, std::string> import_snapshot(const elips::IndexSnapshot& snapshot) override;

private:
    void retrain(size_t n_lists);          // IvfIndexState::rebuild_from_current_data
    void maybe_retrain_after_growth();     // IvfIndexState.cpp:210-230
    void sync_device(bool retrain_codes);  // device index from the host state (+ rebuild_codes)
    void clear();

    elips::Metric metric_;
    std::uint16_t dimension_;
    GpuConfig config_;
    int device_;
    std::uint32_t pq_dim_, pq_bits_;
    size_t requested_lists_, nprobe_;
    elips_b200_ivfpq* h_ = nullptr;
    // IvfIndexState's host state, slot order
    std::vector<RecordID> ids_;
    std::vector<float> host_vectors_;
    std::vector<float> centroids_;
    std::vector<std::uint32_t> assignments_;
    std::unordered_map<RecordID, size_t> slot_of_;
    size_t active_lists_ = 0;
    bool trained_ = false;
    // GpuIVFPQIndex's codebook and codes (read back from the device)
    std::vector<float> codebook_;
    std::vector<std::uint8_t> codes_;
};

// make_gpu_index (GpuHybridIndex.cpp:14-39) with the B200 classes: BruteForce
// and Auto -> B200BruteForceIndex, IvfPq -> B200IvfPqIndex; other algorithms
// (IVF-Flat, the graph) return nullptr: keep the reference's class on the
// CudaBackend port for those.
std::unique_ptr<GpuIndexPort> make_b200_gpu_index(elips::Metric metric, std::uint16_t dimension,
                                                  const GpuConfig& config);

// make_index (IndexFactory.cpp:40-50) with the B200 classes, for a GPU
// policy other than CpuOnly: an exact index with a trained quantizer (a
// quantized vault) and the BruteForce / Auto algorithm -> B200QuantizedIndex;
// otherwise the index make_b200_gpu_index selects. nullptr where the
// reference's own choice stands (CpuOnly, or an algorithm without a B200
// class).
std::unique_ptr<elips::IndexPort> make_b200_index(const elips::Config& config, std::uint16_t dimension);

}  // namespace elips::gpu::b200
