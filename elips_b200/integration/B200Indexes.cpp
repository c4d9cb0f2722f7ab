// Device-resident ELIPS indexes on the B200 library (see B200Indexes.hpp).
#include "B200Indexes.hpp"

#include <algorithm>
#include <cstring>
#include <string_view>
#include <unordered_set>

#include "elips/domain/Errors.hpp"
#include "elips/gpu_engine/GpuIndexTransferManager.hpp"
#include "elips/quant_engine/ProductQuantizer.hpp"
#include "elips/quant_engine/ScalarQuantizer.hpp"
#include "elips_b200.h"

namespace elips::gpu::b200 {
namespace {

GpuError to_error(int status) {
    if (status >= ELIPS_B200_DEVICE_NOT_FOUND && status <= ELIPS_B200_BACKEND_UNAVAILABLE)
        return static_cast<GpuError>(status - 1);
    return GpuError::KernelLaunchFailed;  // dimension mismatch, bad argument, device timeout
}

int device_of(const GpuConfig& config) { return config.device_index < 0 ? 0 : config.device_index; }

// GpuConfig::search_precision -> the library's precision. Auto follows
// enable_fp16_search (GpuConfig.hpp:69); Int8 has no meaning for fp32 rows
// in a brute-force index and keeps fp32.
int precision_of(const GpuConfig& config) {
    switch (config.search_precision) {
        case GpuPrecision::FP16: return ELIPS_B200_PRECISION_FP16;
        case GpuPrecision::FP32: return ELIPS_B200_PRECISION_FP32;
        case GpuPrecision::Int8: return ELIPS_B200_PRECISION_FP32;
        case GpuPrecision::Auto: return config.enable_fp16_search ? ELIPS_B200_PRECISION_FP16 : ELIPS_B200_PRECISION_FP32;
    }
    if (config.search_precision == kGpuPrecisionBF16) return ELIPS_B200_PRECISION_BF16;
    return ELIPS_B200_PRECISION_FP32;
}

void validate_dimension(std::span<const float> v, std::uint16_t dimension, std::string_view label) {
    if (v.size() != dimension)
        throw elips::DimensionMismatch{std::string(label) + " dimension does not match GPU index"};
}

SearchResult result_of(const RecordID& id, float distance) {
    SearchResult r;
    r.id = id;
    r.distance = distance;
    return r;
}

// GpuIVFPQIndex's choose_pq_dim (GpuIVFPQIndex.cpp:24-34): the configured
// pq_dim when it divides the dimension, else the largest divisor <= dim / 8.
std::uint32_t choose_pq_dim(std::uint16_t dimension, std::uint32_t configured) {
    if (configured > 0 && dimension % configured == 0) return configured;
    std::uint32_t guess = std::max<std::uint32_t>(1, dimension / 8);
    while (guess > 1 && dimension % guess != 0) --guess;
    return guess;
}

size_t target_lists(size_t requested, size_t available) {
    return std::max<size_t>(1, std::min(requested, available));
}

}  // namespace

// ===================================================================== exact

B200BruteForceIndex::B200BruteForceIndex(elips::Metric metric, std::uint16_t dimension, const GpuConfig& config)
    : metric_(metric), dimension_(dimension), device_(device_of(config)), precision_(precision_of(config)) {
    reset_device();
}

B200BruteForceIndex::~B200BruteForceIndex() { elips_b200_exact_destroy(h_); }

void B200BruteForceIndex::reset_device() {
    elips_b200_exact_destroy(h_);
    h_ = nullptr;
    const int st = elips_b200_exact_create(device_, static_cast<int>(metric_), precision_, dimension_, &h_);
    if (st != ELIPS_B200_OK) h_ = nullptr;  // searches then return {} / the error, as a failed backend does
}

void B200BruteForceIndex::insert(const RecordID& id, std::span<const float> vector) {
    validate_dimension(vector, dimension_, "vector");
    slot_ids_.push_back(id);
    slot_live_.push_back(1);
    host_vectors_.insert(host_vectors_.end(), vector.begin(), vector.end());
    ++live_;
    if (h_ != nullptr) elips_b200_exact_add(h_, vector.data(), 1);
}

void B200BruteForceIndex::remove(const RecordID& id) {
    // the first live row with this id, as std::find over ids_ (GpuBruteForceIndex.cpp:87-99)
    for (size_t s = 0; s < slot_ids_.size(); ++s) {
        if (slot_live_[s] && slot_ids_[s] == id) {
            slot_live_[s] = 0;
            --live_;
            int removed = 0;
            if (h_ != nullptr) elips_b200_exact_remove(h_, s, &removed);
            compact_if_sparse();
            return;
        }
    }
}

// Removed rows keep their slots until they are half of the index; then the
// device drops them (a stable gather) and the host mirrors follow its map.
void B200BruteForceIndex::compact_if_sparse() {
    if (h_ == nullptr || slot_ids_.size() < 64 || live_ * 2 > slot_ids_.size()) return;
    std::vector<std::uint32_t> new_to_old(std::max<size_t>(1, live_));
    if (elips_b200_exact_compact(h_, new_to_old.data(), new_to_old.size()) != ELIPS_B200_OK) return;
    std::vector<RecordID> ids(live_);
    std::vector<float> vec(live_ * dimension_);
    for (size_t i = 0; i < live_; ++i) {
        ids[i] = slot_ids_[new_to_old[i]];
        std::memcpy(vec.data() + i * dimension_, host_vectors_.data() + size_t{new_to_old[i]} * dimension_,
                    dimension_ * sizeof(float));
    }
    slot_ids_ = std::move(ids);
    host_vectors_ = std::move(vec);
    slot_live_.assign(live_, 1);
}

int B200BruteForceIndex::search_slots(std::span<const float> queries, size_t nq, size_t k, const uint32_t* mask,
                                      std::vector<float>& dist, std::vector<std::int64_t>& slots) const {
    if (h_ == nullptr) return ELIPS_B200_BACKEND_UNAVAILABLE;
    dist.resize(nq * k);
    slots.resize(nq * k);
    return elips_b200_exact_search(h_, queries.data(), nq, k, mask, dist.data(), slots.data());
}

std::vector<IndexPort::Hit> B200BruteForceIndex::search(std::span<const float> query, std::size_t k) const {
    validate_dimension(query, dimension_, "query");
    if (live_ == 0 || k == 0) return {};
    const size_t take = std::min(k, live_);
    std::vector<float> d;
    std::vector<std::int64_t> s;
    if (search_slots(query, 1, take, nullptr, d, s) != ELIPS_B200_OK) return {};  // GpuBruteForceIndex.cpp:112,117
    std::vector<Hit> hits;
    hits.reserve(take);
    for (size_t i = 0; i < take && s[i] >= 0; ++i) hits.emplace_back(slot_ids_[static_cast<size_t>(s[i])], d[i]);
    return hits;
}

std::expected<void, GpuError> B200BruteForceIndex::build_from_batch(std::span<const float> vectors,
                                                                    std::span<const RecordID> ids,
                                                                    const GpuIndexBuildParams&) {
    if (vectors.size() != ids.size() * static_cast<size_t>(dimension_))
        return std::unexpected(GpuError::IndexBuildFailed);
    reset_device();
    if (h_ == nullptr) return std::unexpected(GpuError::InitializationFailed);
    slot_ids_.assign(ids.begin(), ids.end());
    slot_live_.assign(ids.size(), 1);
    host_vectors_.assign(vectors.begin(), vectors.end());
    live_ = ids.size();
    if (!ids.empty()) {
        const int st = elips_b200_exact_add(h_, vectors.data(), ids.size());
        if (st != ELIPS_B200_OK) return std::unexpected(to_error(st));
    }
    return {};
}

std::expected<std::vector<std::vector<SearchResult>>, GpuError>
B200BruteForceIndex::search_batch(std::span<const float> queries, size_t k, size_t) const {
    return search_masked(queries, k, nullptr);
}

std::expected<std::vector<std::vector<SearchResult>>, GpuError>
B200BruteForceIndex::search_batch_filtered(std::span<const float> queries, size_t k,
                                           std::span<const RecordID> candidates) const {
    // MetadataIndex::exact_candidates as a bitmask over this index's slots
    const std::unordered_set<RecordID> want(candidates.begin(), candidates.end());
    std::vector<uint32_t> mask((slot_ids_.size() + 31) / 32, 0u);
    for (size_t s = 0; s < slot_ids_.size(); ++s)
        if (want.contains(slot_ids_[s])) mask[s >> 5] |= 1u << (s & 31);
    return search_masked(queries, k, &mask);
}

std::expected<std::vector<std::vector<SearchResult>>, GpuError>
B200BruteForceIndex::search_masked(std::span<const float> queries, size_t k, const std::vector<uint32_t>* mask) const {
    if (queries.size() % dimension_ != 0) return std::unexpected(GpuError::IndexBuildFailed);
    const size_t nq = queries.size() / dimension_;
    std::vector<std::vector<SearchResult>> out(nq);
    if (live_ == 0 || k == 0 || nq == 0) return out;
    const size_t take = std::min(k, live_);
    std::vector<float> d;
    std::vector<std::int64_t> s;
    const int st = search_slots(queries, nq, take, mask != nullptr ? mask->data() : nullptr, d, s);
    if (st != ELIPS_B200_OK) return std::unexpected(to_error(st));
    for (size_t q = 0; q < nq; ++q) {
        auto& row = out[q];
        row.reserve(take);
        for (size_t i = 0; i < take && s[q * take + i] >= 0; ++i)
            row.push_back(result_of(slot_ids_[static_cast<size_t>(s[q * take + i])], d[q * take + i]));
    }
    return out;
}

std::expected<void, GpuError> B200BruteForceIndex::export_to_cpu_index(elips::IndexPort& cpu_index_out) const {
    auto* transfer = dynamic_cast<elips::IndexTransferPort*>(&cpu_index_out);
    if (transfer == nullptr) return std::unexpected(GpuError::IndexBuildFailed);
    if (!GpuIndexTransferManager::clone_gpu_to_cpu(*this, *transfer).has_value())
        return std::unexpected(GpuError::IndexBuildFailed);
    return {};
}

std::expected<void, GpuError> B200BruteForceIndex::import_from_cpu_index(const elips::IndexPort& cpu_index) {
    const auto* transfer = dynamic_cast<const elips::IndexTransferPort*>(&cpu_index);
    if (transfer == nullptr) return std::unexpected(GpuError::IndexBuildFailed);
    return GpuIndexTransferManager::clone_cpu_to_gpu(*transfer, *this);
}

size_t B200BruteForceIndex::device_bytes_used() const noexcept {
    size_t bytes = 0;
    if (h_ != nullptr) elips_b200_exact_device_bytes(h_, &bytes);
    return bytes;
}

std::expected<elips::IndexSnapshot, std::string> B200BruteForceIndex::export_snapshot() const {
    elips::IndexSnapshot snap;
    snap.kind = elips::IndexSnapshotKind::gpu_brute_force;
    snap.metric = metric_;
    snap.dimension = dimension_;
    snap.ids.reserve(live_);
    snap.vectors.reserve(live_ * dimension_);
    for (size_t s = 0; s < slot_ids_.size(); ++s) {
        if (!slot_live_[s]) continue;
        snap.ids.push_back(slot_ids_[s]);
        snap.vectors.insert(snap.vectors.end(), host_vectors_.begin() + static_cast<std::ptrdiff_t>(s * dimension_),
                            host_vectors_.begin() + static_cast<std::ptrdiff_t>((s + 1) * dimension_));
    }
    return snap;
}

std::expected<void, std::string> B200BruteForceIndex::import_snapshot(const elips::IndexSnapshot& snapshot) {
    if (snapshot.dimension != dimension_) return std::unexpected("snapshot dimension does not match GpuBruteForceIndex");
    if (snapshot.metric != metric_) return std::unexpected("snapshot metric does not match GpuBruteForceIndex");
    if (snapshot.vectors.size() != snapshot.ids.size() * static_cast<size_t>(dimension_))
        return std::unexpected("snapshot vector payload is not row-major brute-force data");
    if (!build_from_batch(snapshot.vectors, snapshot.ids, {}).has_value())
        return std::unexpected("device upload of the snapshot failed");
    return {};
}

// ================================================================ quantized

B200QuantizedIndex::B200QuantizedIndex(elips::Metric metric, std::uint16_t dimension, quant::QuantizerPtr quantizer,
                                       int device)
    : metric_(metric), dimension_(dimension), quantizer_(std::move(quantizer)), device_(device) {
    if (quantizer_ == nullptr) throw std::invalid_argument("B200QuantizedIndex needs a trained quantizer");
    switch (quantizer_->codec()) {
        case quant::CodecId::sq8: {
            const auto* sq = dynamic_cast<const quant::ScalarQuantizer*>(quantizer_.get());
            if (sq == nullptr) throw std::invalid_argument("sq8 codec is not a ScalarQuantizer");
            codec_ = ELIPS_B200_CODEC_SQ8;
            params_ = sq->mins();
            params_.insert(params_.end(), sq->scales().begin(), sq->scales().end());
            break;
        }
        case quant::CodecId::pq:
        case quant::CodecId::opq: {
            const auto* pq = dynamic_cast<const quant::ProductQuantizer*>(quantizer_.get());
            if (pq == nullptr) throw std::invalid_argument("pq codec is not a ProductQuantizer");
            codec_ = pq->codec() == quant::CodecId::opq ? ELIPS_B200_CODEC_OPQ : ELIPS_B200_CODEC_PQ;
            pq_dim_ = static_cast<std::uint32_t>(pq->code_bytes());
            params_ = pq->codebook();
            rotation_ = pq->rotation();
            const size_t per = params_.size() / pq_dim_ / (dimension_ / pq_dim_);
            pq_bits_ = 0;
            while ((size_t{1} << pq_bits_) < per) ++pq_bits_;
            break;
        }
        default:
            throw std::invalid_argument("unsupported codec");
    }
    rebuild_device();
}

B200QuantizedIndex::~B200QuantizedIndex() { elips_b200_quant_destroy(h_); }

void B200QuantizedIndex::rebuild_device() {
    elips_b200_quant_destroy(h_);
    h_ = nullptr;
    if (elips_b200_quant_create(device_, codec_, static_cast<int>(metric_), dimension_, pq_dim_, pq_bits_,
                                params_.data(), rotation_.empty() ? nullptr : rotation_.data(), &h_) != ELIPS_B200_OK) {
        h_ = nullptr;
        return;
    }
    if (!ids_.empty()) elips_b200_quant_add_codes(h_, codes_.data(), ids_.size());
}

void B200QuantizedIndex::insert(const RecordID& id, std::span<const float> vector) {
    if (vector.size() != dimension_) throw elips::DimensionMismatch{"vector dimension does not match index"};
    ids_.push_back(id);
    // Quantizer::encode on the host keeps the host copy the snapshot needs;
    // the device scans the same bytes.
    const auto code = quantizer_->encode(vector);
    codes_.insert(codes_.end(), code.begin(), code.end());
    if (h_ != nullptr) elips_b200_quant_add_codes(h_, code.data(), 1);
}

void B200QuantizedIndex::remove(const RecordID& id) {
    const auto it = std::find(ids_.begin(), ids_.end(), id);
    if (it == ids_.end()) return;
    const size_t row = static_cast<size_t>(it - ids_.begin());
    const size_t w = quantizer_->code_bytes();
    ids_.erase(it);
    codes_.erase(codes_.begin() + static_cast<std::ptrdiff_t>(row * w),
                 codes_.begin() + static_cast<std::ptrdiff_t>((row + 1) * w));
    rebuild_device();  // the codes are small (code_bytes per row): re-upload in order
}

std::vector<IndexPort::Hit> B200QuantizedIndex::search(std::span<const float> query, std::size_t k) const {
    if (query.size() != dimension_) throw elips::DimensionMismatch{"query dimension does not match index"};
    if (ids_.empty() || k == 0 || h_ == nullptr) return {};
    const size_t take = std::min(k, ids_.size());
    std::vector<float> d(take);
    std::vector<std::int64_t> r(take);
    if (elips_b200_quant_search(h_, query.data(), 1, take, d.data(), r.data()) != ELIPS_B200_OK) return {};
    std::vector<Hit> hits;
    for (size_t i = 0; i < take && r[i] >= 0; ++i) hits.emplace_back(ids_[static_cast<size_t>(r[i])], d[i]);
    return hits;
}

std::expected<elips::IndexSnapshot, std::string> B200QuantizedIndex::export_snapshot() const {
    // ExactIndex::export_snapshot (ExactIndex.cpp:89-116): fp32 vectors decoded
    // from the codes, the codes riding along in `pq`.
    elips::IndexSnapshot snap;
    snap.kind = elips::IndexSnapshotKind::exact;
    snap.metric = metric_;
    snap.dimension = dimension_;
    snap.ids = ids_;
    const size_t w = quantizer_->code_bytes();
    snap.vectors.resize(ids_.size() * dimension_);
    for (size_t i = 0; i < ids_.size(); ++i)
        quantizer_->decode(std::span<const std::uint8_t>{codes_.data() + i * w, w},
                           std::span<float>{snap.vectors}.subspan(i * dimension_, dimension_));
    elips::PqSnapshot pq;
    pq.codec = quantizer_->codec();
    pq.pq_dim = static_cast<std::uint32_t>(w);
    pq.codes = codes_;
    snap.pq = std::move(pq);
    return snap;
}

std::expected<void, std::string> B200QuantizedIndex::import_snapshot(const elips::IndexSnapshot& snapshot) {
    if (snapshot.dimension != dimension_) return std::unexpected("snapshot dimension does not match ExactIndex");
    if (snapshot.metric != metric_) return std::unexpected("snapshot metric does not match ExactIndex");
    if (snapshot.vectors.size() != snapshot.ids.size() * static_cast<size_t>(dimension_))
        return std::unexpected("snapshot vector payload is not row-major exact data");
    // re-encoded from the fp32 payload, as ExactIndex::import_snapshot does
    ids_ = snapshot.ids;
    codes_.clear();
    codes_.reserve(ids_.size() * quantizer_->code_bytes());
    for (size_t i = 0; i < ids_.size(); ++i) {
        const auto code = quantizer_->encode(
            std::span<const float>{snapshot.vectors.data() + i * dimension_, dimension_});
        codes_.insert(codes_.end(), code.begin(), code.end());
    }
    rebuild_device();
    return {};
}

// ==================================================================== IVF-PQ

B200IvfPqIndex::B200IvfPqIndex(elips::Metric metric, std::uint16_t dimension, const GpuConfig& config)
    : metric_(metric),
      dimension_(dimension),
      config_(config),
      device_(device_of(config)),
      pq_dim_(choose_pq_dim(dimension, config.ivf_pq_params.pq_dim)),
      pq_bits_(std::clamp<std::uint32_t>(config.ivf_pq_params.pq_bits, 4U, 8U)),
      requested_lists_(std::max<size_t>(1, config.ivf_pq_params.n_lists)),
      nprobe_(std::max<size_t>(1, config.default_ef_search_gpu)) {}

B200IvfPqIndex::~B200IvfPqIndex() { elips_b200_ivfpq_destroy(h_); }

void B200IvfPqIndex::clear() {
    ids_.clear();
    host_vectors_.clear();
    centroids_.clear();
    assignments_.clear();
    slot_of_.clear();
    codebook_.clear();
    codes_.clear();
    active_lists_ = 0;
    trained_ = false;
    elips_b200_ivfpq_destroy(h_);
    h_ = nullptr;
}

// IvfIndexState::rebuild_from_current_data (IvfIndexState.cpp:193-208):
// train_centroids + the final assignment, on the device, bit-identical.
void B200IvfPqIndex::retrain(size_t n_lists) {
    active_lists_ = target_lists(n_lists, ids_.size());
    centroids_.assign(active_lists_ * dimension_, 0.0f);
    assignments_.assign(ids_.size(), 0u);
    const int st = elips_b200_ivf_train(device_, static_cast<int>(metric_), host_vectors_.data(), ids_.size(),
                                        dimension_, active_lists_,
                                        std::max<size_t>(1, config_.ivf_pq_params.kmeans_n_iters), centroids_.data(),
                                        assignments_.data(), 0, nullptr);
    trained_ = st == ELIPS_B200_OK;
}

// IvfIndexState::maybe_retrain_after_growth (IvfIndexState.cpp:210-230)
void B200IvfPqIndex::maybe_retrain_after_growth() {
    const size_t target = target_lists(requested_lists_, ids_.size());
    if (!trained_) {
        retrain(target);
        return;
    }
    if (target > active_lists_ && (target == requested_lists_ || ids_.size() >= active_lists_ * 2)) retrain(target);
}

// The device index from the host state. retrain_codes = GpuIVFPQIndex::
// rebuild_codes (GpuIVFPQIndex.cpp:88-130): a new codebook trained on every
// residual and every row re-encoded, on the device; otherwise the codebook
// and codes held (a snapshot's) are imported as given.
void B200IvfPqIndex::sync_device(bool retrain_codes) {
    elips_b200_ivfpq_destroy(h_);
    h_ = nullptr;
    if (ids_.empty() || !trained_) {
        codebook_.clear();
        codes_.clear();
        return;
    }
    const size_t ksub = size_t{1} << pq_bits_;
    if (retrain_codes || codebook_.size() != pq_dim_ * ksub * (dimension_ / pq_dim_))
        codebook_.assign(pq_dim_ * ksub * (dimension_ / pq_dim_), 0.0f);
    if (elips_b200_ivfpq_create(device_, static_cast<int>(metric_), dimension_, static_cast<uint32_t>(active_lists_),
                                static_cast<uint32_t>(nprobe_), pq_dim_, pq_bits_, centroids_.data(),
                                codebook_.data(), &h_) != ELIPS_B200_OK) {
        h_ = nullptr;
        return;
    }
    const bool have_codes = !retrain_codes && codes_.size() == ids_.size() * pq_dim_;
    if (elips_b200_ivfpq_add(h_, host_vectors_.data(), assignments_.data(), have_codes ? codes_.data() : nullptr,
                             ids_.size()) != ELIPS_B200_OK) {
        elips_b200_ivfpq_destroy(h_);
        h_ = nullptr;
        return;
    }
    if (!have_codes) {
        if (elips_b200_ivfpq_rebuild_codes(h_) != ELIPS_B200_OK) return;
        // read back the model the device now holds (the snapshot carries it)
        std::vector<float> cent(active_lists_ * dimension_);
        std::vector<std::uint32_t> asg(ids_.size());
        std::vector<float> vec(ids_.size() * dimension_);
        codes_.assign(ids_.size() * pq_dim_, 0);
        elips_b200_ivfpq_export(h_, cent.data(), asg.data(), vec.data(), codebook_.data(), codes_.data());
    }
}

void B200IvfPqIndex::insert(const RecordID& id, std::span<const float> vector) {
    validate_dimension(vector, dimension_, "vector");
    // IvfIndexState::insert (IvfIndexState.cpp:232-262): an id present already is replaced
    if (slot_of_.contains(id)) {
        remove(id);
    }
    ids_.push_back(id);
    host_vectors_.insert(host_vectors_.end(), vector.begin(), vector.end());
    slot_of_[id] = ids_.size() - 1;
    if (trained_) {
        std::uint32_t list = 0;
        elips_b200_ivf_assign(device_, static_cast<int>(metric_), vector.data(), 1, dimension_, centroids_.data(),
                              active_lists_, &list, nullptr, 0, nullptr);
        assignments_.push_back(list);
    }
    maybe_retrain_after_growth();
    sync_device(true);  // GpuIVFPQIndex::insert then rebuild_codes (GpuIVFPQIndex.cpp:150-154)
}

void B200IvfPqIndex::remove(const RecordID& id) {
    // IvfIndexState::remove (IvfIndexState.cpp:262-326): the last slot moves
    // into the removed one, list member order kept
    const auto found = slot_of_.find(id);
    if (found == slot_of_.end()) return;
    const size_t slot = found->second, last = ids_.size() - 1;
    if (slot != last) {
        ids_[slot] = ids_[last];
        std::copy(host_vectors_.begin() + static_cast<std::ptrdiff_t>(last * dimension_),
                  host_vectors_.begin() + static_cast<std::ptrdiff_t>((last + 1) * dimension_),
                  host_vectors_.begin() + static_cast<std::ptrdiff_t>(slot * dimension_));
        slot_of_[ids_[slot]] = slot;
        if (trained_) assignments_[slot] = assignments_[last];
    }
    ids_.pop_back();
    host_vectors_.resize(ids_.size() * dimension_);
    slot_of_.erase(found);
    if (trained_ && !assignments_.empty()) assignments_.pop_back();
    if (ids_.empty()) {
        clear();
        return;
    }
    if (trained_ && active_lists_ > ids_.size()) retrain(ids_.size());
    sync_device(true);  // GpuIVFPQIndex::remove then rebuild_codes (GpuIVFPQIndex.cpp:156-159)
}

std::vector<IndexPort::Hit> B200IvfPqIndex::search(std::span<const float> query, std::size_t k) const {
    validate_dimension(query, dimension_, "query");
    if (ids_.empty() || k == 0 || h_ == nullptr) return {};
    std::vector<float> d(k);
    std::vector<std::int64_t> r(k);
    if (elips_b200_ivfpq_search(h_, query.data(), 1, k, d.data(), r.data()) != ELIPS_B200_OK) return {};
    std::vector<Hit> hits;
    for (size_t i = 0; i < k && r[i] >= 0; ++i) hits.emplace_back(ids_[static_cast<size_t>(r[i])], d[i]);
    return hits;
}

std::expected<void, GpuError> B200IvfPqIndex::build_from_batch(std::span<const float> vectors,
                                                               std::span<const RecordID> ids,
                                                               const GpuIndexBuildParams&) {
    if (vectors.size() != ids.size() * static_cast<size_t>(dimension_))
        return std::unexpected(GpuError::IndexBuildFailed);
    clear();
    if (ids.empty()) return {};
    ids_.assign(ids.begin(), ids.end());
    host_vectors_.assign(vectors.begin(), vectors.end());
    for (size_t i = 0; i < ids_.size(); ++i) slot_of_[ids_[i]] = i;
    // IvfIndexState::build_from_batch + rebuild_codes, in one device call
    active_lists_ = target_lists(requested_lists_, ids_.size());
    centroids_.assign(active_lists_ * dimension_, 0.0f);
    assignments_.assign(ids_.size(), 0u);
    codebook_.assign(pq_dim_ * (size_t{1} << pq_bits_) * (dimension_ / pq_dim_), 0.0f);
    codes_.assign(ids_.size() * pq_dim_, 0);
    const int st = elips_b200_ivfpq_train(device_, static_cast<int>(metric_), host_vectors_.data(), ids_.size(),
                                          dimension_, active_lists_,
                                          std::max<size_t>(1, config_.ivf_pq_params.kmeans_n_iters), pq_dim_,
                                          pq_bits_, centroids_.data(), assignments_.data(), codebook_.data(),
                                          codes_.data(), 0, nullptr);
    if (st != ELIPS_B200_OK) return std::unexpected(GpuError::IndexBuildFailed);
    trained_ = true;
    sync_device(false);
    if (h_ == nullptr) return std::unexpected(GpuError::IndexBuildFailed);
    return {};
}

std::expected<std::vector<std::vector<SearchResult>>, GpuError>
B200IvfPqIndex::search_batch(std::span<const float> queries, size_t k, size_t) const {
    if (queries.size() % dimension_ != 0) return std::unexpected(GpuError::IndexBuildFailed);
    const size_t nq = queries.size() / dimension_;
    std::vector<std::vector<SearchResult>> out(nq);
    if (ids_.empty() || k == 0 || nq == 0) return out;
    if (h_ == nullptr) return std::unexpected(GpuError::BackendUnavailable);
    std::vector<float> d(nq * k);
    std::vector<std::int64_t> r(nq * k);
    const int st = elips_b200_ivfpq_search(h_, queries.data(), nq, k, d.data(), r.data());
    if (st != ELIPS_B200_OK) return std::unexpected(to_error(st));
    for (size_t q = 0; q < nq; ++q)
        for (size_t i = 0; i < k && r[q * k + i] >= 0; ++i)
            out[q].push_back(result_of(ids_[static_cast<size_t>(r[q * k + i])], d[q * k + i]));
    return out;
}

std::expected<void, GpuError> B200IvfPqIndex::export_to_cpu_index(elips::IndexPort& cpu_index_out) const {
    auto* transfer = dynamic_cast<elips::IndexTransferPort*>(&cpu_index_out);
    if (transfer == nullptr) return std::unexpected(GpuError::IndexBuildFailed);
    if (!GpuIndexTransferManager::clone_gpu_to_cpu(*this, *transfer).has_value())
        return std::unexpected(GpuError::IndexBuildFailed);
    return {};
}

std::expected<void, GpuError> B200IvfPqIndex::import_from_cpu_index(const elips::IndexPort& cpu_index) {
    const auto* transfer = dynamic_cast<const elips::IndexTransferPort*>(&cpu_index);
    if (transfer == nullptr) return std::unexpected(GpuError::IndexBuildFailed);
    return GpuIndexTransferManager::clone_cpu_to_gpu(*transfer, *this);
}

size_t B200IvfPqIndex::device_bytes_used() const noexcept {
    // raw rows (rerank), codes in slot order and list-major, list members,
    // centroids and codebook
    return host_vectors_.size() * sizeof(float) + codes_.size() * 2 + ids_.size() * 8 +
           centroids_.size() * sizeof(float) + codebook_.size() * sizeof(float);
}

std::expected<elips::IndexSnapshot, std::string> B200IvfPqIndex::export_snapshot() const {
    // IvfIndexState::export_snapshot + GpuIVFPQIndex's pq section (:306-318)
    elips::IndexSnapshot snap;
    snap.kind = elips::IndexSnapshotKind::gpu_ivf_pq;
    snap.metric = metric_;
    snap.dimension = dimension_;
    snap.ids = ids_;
    snap.vectors = host_vectors_;
    if (trained_ && active_lists_ > 0) {
        elips::IvfSnapshot ivf;
        ivf.n_lists = active_lists_;
        ivf.n_probe = nprobe_;
        ivf.centroids = centroids_;
        ivf.assignments = assignments_;
        snap.ivf = std::move(ivf);
    }
    if (!codebook_.empty()) {
        elips::PqSnapshot pq;
        pq.pq_dim = pq_dim_;
        pq.pq_bits = pq_bits_;
        pq.codebook = codebook_;
        pq.codes = codes_;
        snap.pq = std::move(pq);
    }
    return snap;
}

std::expected<void, std::string> B200IvfPqIndex::import_snapshot(const elips::IndexSnapshot& snapshot) {
    // GpuIVFPQIndex::import_snapshot (:327-348) over IvfIndexState::import_snapshot (:339-374)
    if (snapshot.dimension != dimension_) return std::unexpected("snapshot dimension does not match IVF index");
    if (snapshot.metric != metric_) return std::unexpected("snapshot metric does not match IVF index");
    if (snapshot.vectors.size() != snapshot.ids.size() * static_cast<size_t>(dimension_))
        return std::unexpected("snapshot vector payload is not row-major IVF data");
    clear();
    if (snapshot.pq.has_value()) {
        pq_dim_ = snapshot.pq->pq_dim;
        pq_bits_ = snapshot.pq->pq_bits;
        codebook_ = snapshot.pq->codebook;
        codes_ = snapshot.pq->codes;
    }
    ids_ = snapshot.ids;
    host_vectors_ = snapshot.vectors;
    for (size_t i = 0; i < ids_.size(); ++i) slot_of_[ids_[i]] = i;
    if (snapshot.ivf.has_value() && snapshot.ivf->centroids.size() == snapshot.ivf->n_lists * dimension_ &&
        snapshot.ivf->assignments.size() == ids_.size()) {
        active_lists_ = target_lists(snapshot.ivf->n_lists, ids_.size());
        nprobe_ = std::max<size_t>(1, snapshot.ivf->n_probe);
        centroids_ = snapshot.ivf->centroids;
        centroids_.resize(active_lists_ * dimension_);
        assignments_ = snapshot.ivf->assignments;
        trained_ = !ids_.empty();
    } else if (!ids_.empty()) {
        retrain(target_lists(requested_lists_, ids_.size()));
    }
    const bool codes_ok = !codebook_.empty() && codes_.size() == ids_.size() * pq_dim_;
    sync_device(!codes_ok);
    if (!ids_.empty() && h_ == nullptr) return std::unexpected("device upload of the snapshot failed");
    return {};
}

// ================================================================= selection

std::unique_ptr<GpuIndexPort> make_b200_gpu_index(elips::Metric metric, std::uint16_t dimension,
                                                  const GpuConfig& config) {
    switch (config.algorithm) {
        case GpuIndexAlgorithm::BruteForce:
        case GpuIndexAlgorithm::Auto:
            return std::make_unique<B200BruteForceIndex>(metric, dimension, config);
        case GpuIndexAlgorithm::IvfPq:
            return std::make_unique<B200IvfPqIndex>(metric, dimension, config);
        default:
            return nullptr;
    }
}

std::unique_ptr<elips::IndexPort> make_b200_index(const elips::Config& config, std::uint16_t dimension) {
    if (!config.has_gpu() || config.gpu().policy == GpuPolicy::CpuOnly) return nullptr;
    const auto algo = config.gpu().algorithm;
    // a quantized vault's exact scan (ExactIndex with its Quantizer) on the device
    if (config.index() == elips::IndexType::exact && config.quantizer() != nullptr &&
        (algo == GpuIndexAlgorithm::BruteForce || algo == GpuIndexAlgorithm::Auto))
        return std::make_unique<B200QuantizedIndex>(config.metric(), dimension, config.quantizer(),
                                                    device_of(config.gpu()));
    return make_b200_gpu_index(config.metric(), dimension, config.gpu());
}

}  // namespace elips::gpu::b200
