// Test infrastructure only: a C-ABI driver over the reference's own compiled
// classes (ExactIndex, ScalarQuantizer, ProductQuantizer, quant::detail
// k-means, GpuIVFPQIndex / GpuIVFFlatIndex / GpuBruteForceIndex on a GpuPort).
// It is linked with the reference sources by oracle/Makefile into
// oracle/_ref/libelips_ref.so (a CPU GpuPort), and is used by the tests to pin
// the C restatement in oracle/oracle.c, to generate golden fixtures, and by
// bench.py's CPU baseline / reference arm. Nothing in the product path loads
// it. Built with REF_WITH_B200 (oracle/_ref/libelips_ref_b200.so) it can also
// run those reference classes on elips::gpu::cuda::CudaBackend
// (elips_b200/integration/CudaBackend.cpp): the drop-in check of the GpuPort
// boundary.
//
// Row identity: every row i is given RecordID(bytes) whose last eight bytes are
// i in big-endian order, so search results map back to row indexes
// deterministically (RecordID.hpp:18 takes raw bytes).

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <span>
#include <thread>
#include <vector>

#include "elips/Config.hpp"
#include "elips/domain/RecordID.hpp"
#include "elips/domain/Vector.hpp"
#include "elips/gpu_engine/GpuBruteForceIndex.hpp"
#include "elips/gpu_engine/GpuIVFFlatIndex.hpp"
#include "elips/gpu_engine/GpuIVFPQIndex.hpp"
#include "elips/gpu_engine/GpuPort.hpp"
#include "elips/index_engine/ExactIndex.hpp"
#include "elips/index_engine/IndexSnapshot.hpp"
#include "elips/quant_engine/ProductQuantizer.hpp"
#include "elips/quant_engine/ScalarQuantizer.hpp"
#include "elips/quant_engine/detail/KMeans.hpp"
#include "elips/vector_engine/Metrics.hpp"
#ifdef REF_WITH_B200
#include "B200Indexes.hpp"
#include "backends/cuda/CudaBackend.hpp"
#include "elips/domain/Errors.hpp"
#endif

namespace {

using elips::Metric;
using elips::RecordID;

RecordID row_id(std::uint64_t row) {
    RecordID::Bytes b{};
    for (int i = 0; i < 8; ++i) {
        b[15 - i] = static_cast<std::uint8_t>(row >> (8 * i));
    }
    return RecordID{b};
}

std::int64_t id_row(const RecordID& id) {
    std::uint64_t row = 0;
    for (int i = 8; i < 16; ++i) {
        row = (row << 8) | id.bytes()[i];
    }
    return static_cast<std::int64_t>(row);
}

// A stateless, thread-safe CPU GpuPort: compute_distances_batch is the
// reference distance loop and top_k is a partial_sort, the same arithmetic as
// the reference's own test backend (tests/unit/gpu/TestRecordingBackend.hpp:
// 75-120). Ties in top_k break by index so repeated runs agree.
class CpuPort final : public elips::gpu::GpuPort {
public:
    std::expected<void, elips::gpu::GpuError> initialize(const elips::gpu::GpuConfig&) override { return {}; }
    void shutdown() noexcept override {}
    elips::gpu::GpuDeviceInfo device_info() const noexcept override {
        elips::gpu::GpuDeviceInfo info;
        info.name = "cpu-oracle";
        info.backend = "cpu";
        info.supports_ivf_pq = true;
        return info;
    }
    bool is_available() const noexcept override { return true; }
    std::expected<elips::gpu::GpuBuffer, elips::gpu::GpuError> allocate_device(size_t bytes) override {
        return elips::gpu::GpuBuffer{nullptr, bytes, this};
    }
    void free_device(elips::gpu::GpuBuffer) noexcept override {}
    std::expected<void, elips::gpu::GpuError> upload(const void*, elips::gpu::GpuBuffer&, size_t) override { return {}; }
    std::expected<void, elips::gpu::GpuError> download(const elips::gpu::GpuBuffer&, void*, size_t) override { return {}; }
    std::expected<void, elips::gpu::GpuError> compute_distances_batch(
        std::span<const float> queries, std::span<const float> database,
        std::span<float> out, size_t nq, size_t nb, size_t dim, Metric metric) override {
        for (size_t q = 0; q < nq; ++q) {
            const auto query = queries.subspan(q * dim, dim);
            for (size_t i = 0; i < nb; ++i) {
                out[q * nb + i] = elips::distance(metric, query, database.subspan(i * dim, dim));
            }
        }
        return {};
    }
    std::expected<void, elips::gpu::GpuError> top_k(
        std::span<const float> distances, std::span<uint32_t> indices_out,
        std::span<float> values_out, size_t nq, size_t nb, size_t k) override {
        for (size_t q = 0; q < nq; ++q) {
            std::vector<std::pair<float, uint32_t>> ranked(nb);
            for (size_t i = 0; i < nb; ++i) {
                ranked[i] = {distances[q * nb + i], static_cast<uint32_t>(i)};
            }
            const auto take = std::min(k, nb);
            std::partial_sort(ranked.begin(), ranked.begin() + static_cast<std::ptrdiff_t>(take),
                              ranked.end());
            for (size_t i = 0; i < take; ++i) {
                indices_out[q * k + i] = ranked[i].second;
                values_out[q * k + i] = ranked[i].first;
            }
        }
        return {};
    }
    void synchronize() override {}
    bool is_idle() const noexcept override { return true; }
};

// Runs fn(q) for q in [0, nq) on nthreads std::threads (strided split).
template <class Fn>
void parallel_queries(size_t nq, int nthreads, Fn fn) {
    if (nthreads <= 1 || nq <= 1) {
        for (size_t q = 0; q < nq; ++q) fn(q);
        return;
    }
    const size_t workers = std::min<size_t>(static_cast<size_t>(nthreads), nq);
    std::vector<std::thread> pool;
    pool.reserve(workers);
    for (size_t w = 0; w < workers; ++w) {
        pool.emplace_back([&, w] {
            for (size_t q = w; q < nq; q += workers) fn(q);
        });
    }
    for (auto& t : pool) t.join();
}

template <class Hit>
void write_hits(const std::vector<Hit>& hits, size_t k, float* out_dist, std::int64_t* out_rows) {
    for (size_t i = 0; i < k; ++i) {
        if (i < hits.size()) {
            out_dist[i] = hits[i].second;
            out_rows[i] = id_row(hits[i].first);
        } else {
            out_dist[i] = 0.0F;
            out_rows[i] = -1;
        }
    }
}

struct ExactHandle {
    std::unique_ptr<elips::ExactIndex> index;
};

// The GpuPort the next index handle is built on: the CPU port, or (in the
// REF_WITH_B200 build, after ref_use_b200_port(1)) the B200 CudaBackend.
std::atomic<int> g_use_b200{0};

std::unique_ptr<elips::gpu::GpuPort> make_port() {
#ifdef REF_WITH_B200
    if (g_use_b200.load()) {
        auto port = std::make_unique<elips::gpu::cuda::CudaBackend>();
        elips::gpu::GpuConfig config;
        config.device_index = 0;
        if (!port->initialize(config).has_value()) return nullptr;
        return port;
    }
#endif
    return std::make_unique<CpuPort>();
}

struct IvfPqHandle {
    std::unique_ptr<elips::gpu::GpuPort> port = make_port();
    std::unique_ptr<elips::gpu::GpuIVFPQIndex> index;
};

struct IvfFlatHandle {
    std::unique_ptr<elips::gpu::GpuPort> port = make_port();
    std::unique_ptr<elips::gpu::GpuIVFFlatIndex> index;
};

struct BruteHandle {
    std::unique_ptr<elips::gpu::GpuPort> port = make_port();
    std::unique_ptr<elips::gpu::GpuBruteForceIndex> index;
};

}  // namespace

extern "C" {

// Vector::normalized (Vector.hpp:34-44) of every row.
void ref_normalize_rows(const float* in, float* out, size_t n, size_t d) {
    for (size_t r = 0; r < n; ++r) {
        const elips::Vector v{std::vector<float>(in + r * d, in + (r + 1) * d)};
        const auto out_v = v.normalized();
        std::copy(out_v.values().begin(), out_v.values().end(), out + r * d);
    }
}

float ref_distance(int metric, const float* a, const float* b, size_t n) {
    return elips::distance(static_cast<Metric>(metric), std::span<const float>{a, n},
                           std::span<const float>{b, n});
}

// ExactIndex over fp32 rows (no quantizer).
void* ref_exact_create(int metric, uint32_t dim, const float* rows, size_t n) {
    auto* h = new ExactHandle;
    h->index = std::make_unique<elips::ExactIndex>(static_cast<Metric>(metric),
                                                   static_cast<std::uint16_t>(dim));
    for (size_t i = 0; i < n; ++i) {
        h->index->insert(row_id(i), std::span<const float>{rows + i * dim, dim});
    }
    return h;
}

// ExactIndex with the reference's sq8 codec built from given mins/scales; the
// rows are encoded by the reference's own ScalarQuantizer::encode.
void* ref_sq8_exact_create(int metric, uint32_t dim, const float* mins, const float* scales,
                           const float* rows, size_t n) {
    auto q = std::make_shared<elips::quant::ScalarQuantizer>(
        static_cast<Metric>(metric), static_cast<std::uint16_t>(dim),
        std::vector<float>(mins, mins + dim), std::vector<float>(scales, scales + dim));
    auto* h = new ExactHandle;
    h->index = std::make_unique<elips::ExactIndex>(static_cast<Metric>(metric),
                                                   static_cast<std::uint16_t>(dim), q);
    for (size_t i = 0; i < n; ++i) {
        h->index->insert(row_id(i), std::span<const float>{rows + i * dim, dim});
    }
    return h;
}

// ExactIndex with a plain (non-residual, no rotation) PQ codec built from a
// given codebook [pq_dim][2^pq_bits][dim/pq_dim].
void* ref_pq_exact_create(int metric, uint32_t dim, uint32_t pq_dim, uint32_t pq_bits,
                          const float* codebook, const float* rows, size_t n) {
    const size_t cb = static_cast<size_t>(pq_dim) * (size_t{1} << pq_bits) * (dim / pq_dim);
    auto q = std::make_shared<elips::quant::ProductQuantizer>(
        static_cast<Metric>(metric), static_cast<std::uint16_t>(dim), pq_dim, pq_bits,
        std::vector<float>(codebook, codebook + cb), std::vector<float>{});
    auto* h = new ExactHandle;
    h->index = std::make_unique<elips::ExactIndex>(static_cast<Metric>(metric),
                                                   static_cast<std::uint16_t>(dim), q);
    for (size_t i = 0; i < n; ++i) {
        h->index->insert(row_id(i), std::span<const float>{rows + i * dim, dim});
    }
    return h;
}

// ExactIndex with an OPQ codec (ProductQuantizer with a rotation) built from
// a given codebook and dimension x dimension rotation.
void* ref_opq_exact_create(int metric, uint32_t dim, uint32_t pq_dim, uint32_t pq_bits,
                           const float* codebook, const float* rotation, const float* rows, size_t n) {
    const size_t cb = static_cast<size_t>(pq_dim) * (size_t{1} << pq_bits) * (dim / pq_dim);
    auto q = std::make_shared<elips::quant::ProductQuantizer>(
        static_cast<Metric>(metric), static_cast<std::uint16_t>(dim), pq_dim, pq_bits,
        std::vector<float>(codebook, codebook + cb),
        std::vector<float>(rotation, rotation + static_cast<size_t>(dim) * dim));
    auto* h = new ExactHandle;
    h->index = std::make_unique<elips::ExactIndex>(static_cast<Metric>(metric),
                                                   static_cast<std::uint16_t>(dim), q);
    for (size_t i = 0; i < n; ++i) {
        h->index->insert(row_id(i), std::span<const float>{rows + i * dim, dim});
    }
    return h;
}

int ref_exact_search(void* handle, uint32_t dim, const float* queries, size_t nq, size_t k,
                     int nthreads, float* out_dist, std::int64_t* out_rows) {
    auto* h = static_cast<ExactHandle*>(handle);
    parallel_queries(nq, nthreads, [&](size_t q) {
        const auto hits = h->index->search(std::span<const float>{queries + q * dim, dim}, k);
        write_hits(hits, k, out_dist + q * k, out_rows + q * k);
    });
    return 0;
}

void ref_exact_destroy(void* handle) { delete static_cast<ExactHandle*>(handle); }

// ScalarQuantizer::train (ScalarQuantizer.cpp:26-50).
void ref_sq8_train(int metric, uint32_t dim, const float* rows, size_t n, float* mins_out,
                   float* scales_out) {
    auto q = elips::quant::ScalarQuantizer::train(static_cast<Metric>(metric),
                                                  static_cast<std::uint16_t>(dim),
                                                  std::span<const float>{rows, n * dim}, n);
    std::copy(q->mins().begin(), q->mins().end(), mins_out);
    std::copy(q->scales().begin(), q->scales().end(), scales_out);
}

// ScalarQuantizer::encode over n rows (ScalarQuantizer.cpp:52-68).
void ref_sq8_encode(int metric, uint32_t dim, const float* mins, const float* scales,
                    const float* rows, size_t n, std::uint8_t* codes_out) {
    elips::quant::ScalarQuantizer q(static_cast<Metric>(metric), static_cast<std::uint16_t>(dim),
                                    std::vector<float>(mins, mins + dim),
                                    std::vector<float>(scales, scales + dim));
    for (size_t i = 0; i < n; ++i) {
        q.encode(std::span<const float>{rows + i * dim, dim},
                 std::span<std::uint8_t>{codes_out + i * dim, dim});
    }
}

// ScalarQuantizer::make_lut + lut_distance for one query over n codes.
void ref_sq8_distances(int metric, uint32_t dim, const float* mins, const float* scales,
                       const float* query, const std::uint8_t* codes, size_t n, float* out) {
    elips::quant::ScalarQuantizer q(static_cast<Metric>(metric), static_cast<std::uint16_t>(dim),
                                    std::vector<float>(mins, mins + dim),
                                    std::vector<float>(scales, scales + dim));
    const auto lut = q.make_lut(std::span<const float>{query, dim});
    for (size_t i = 0; i < n; ++i) {
        out[i] = q.lut_distance(lut, std::span<const std::uint8_t>{codes + i * dim, dim});
    }
}

// quant::detail::train_pq_codebook (KMeans.cpp:249-268).
void ref_train_pq_codebook(const float* rows, size_t n, size_t dim, size_t pq_dim, size_t ksub,
                           size_t iters, float* codebook_out) {
    elips::quant::detail::train_pq_codebook(
        std::span<const float>{rows, n * dim}, n, dim, pq_dim, ksub, iters,
        std::span<float>{codebook_out, pq_dim * ksub * (dim / pq_dim)});
}

// quant::detail::encode_pq (KMeans.cpp:270-285).
void ref_encode_pq(const float* rows, const float* codebook, size_t n, size_t dim, size_t pq_dim,
                   size_t ksub, std::uint8_t* codes_out) {
    elips::quant::detail::encode_pq(
        std::span<const float>{rows, n * dim},
        std::span<const float>{codebook, pq_dim * ksub * (dim / pq_dim)}, n, dim, pq_dim, ksub,
        std::span<std::uint8_t>{codes_out, n * pq_dim});
}

// IvfIndexState::train_centroids + assign_vectors_to_centroids, run by
// GpuIVFFlatIndex::build_from_batch on the CPU port and read back through
// export_snapshot (IvfIndexState.cpp:118-208, 328-337).
int ref_ivf_train(int metric, uint32_t dim, const float* rows, size_t n, size_t n_lists, size_t iters,
                  float* centroids_out, uint32_t* assignments_out) {
    CpuPort port;
    elips::gpu::GpuConfig config;
    config.ivf_pq_params.n_lists = n_lists;
    config.ivf_pq_params.kmeans_n_iters = iters;
    elips::gpu::GpuIVFFlatIndex index(port, static_cast<Metric>(metric), static_cast<std::uint16_t>(dim), config);
    std::vector<RecordID> ids;
    ids.reserve(n);
    for (size_t i = 0; i < n; ++i) ids.push_back(row_id(i));
    if (!index.build_from_batch(std::span<const float>{rows, n * dim}, ids, {}).has_value()) return 1;
    const auto snap = index.export_snapshot();
    if (!snap.has_value() || !snap->ivf.has_value()) return 2;
    const auto& ivf = *snap->ivf;
    if (ivf.centroids.size() != n_lists * dim || ivf.assignments.size() != n) return 3;
    std::copy(ivf.centroids.begin(), ivf.centroids.end(), centroids_out);
    std::copy(ivf.assignments.begin(), ivf.assignments.end(), assignments_out);
    return 0;
}

// quant::detail::kmeans (KMeans.cpp:182-247).
void ref_kmeans(const float* rows, size_t n, size_t dim, size_t k, size_t iters,
                float* centroids_out) {
    elips::quant::detail::kmeans(std::span<const float>{rows, n * dim}, n, dim, k, iters,
                                 std::span<float>{centroids_out, k * dim});
}

// ProductQuantizer::make_lut + lut_distance for one query over n codes.
void ref_pq_distances(int metric, uint32_t dim, uint32_t pq_dim, uint32_t pq_bits,
                      const float* codebook, const float* query, const std::uint8_t* codes,
                      size_t n, float* out) {
    const size_t cb = static_cast<size_t>(pq_dim) * (size_t{1} << pq_bits) * (dim / pq_dim);
    elips::quant::ProductQuantizer q(static_cast<Metric>(metric), static_cast<std::uint16_t>(dim),
                                     pq_dim, pq_bits, std::vector<float>(codebook, codebook + cb),
                                     std::vector<float>{});
    const auto lut = q.make_lut(std::span<const float>{query, dim});
    for (size_t i = 0; i < n; ++i) {
        out[i] = q.lut_distance(lut, std::span<const std::uint8_t>{codes + i * pq_dim, pq_dim});
    }
}

// GpuIVFPQIndex on the CPU port, loaded through import_snapshot with a model
// trained elsewhere (GpuIVFPQIndex.cpp:327-348, IvfIndexState.cpp:339-374).
// codes are the residual PQ codes, one pq_dim-byte row per vector.
void* ref_ivfpq_create(int metric, uint32_t dim, size_t n_lists, size_t nprobe, uint32_t pq_dim,
                       uint32_t pq_bits, const float* centroids, const uint32_t* assignments,
                       const float* codebook, const std::uint8_t* codes, const float* vectors,
                       size_t n) {
    auto* h = new IvfPqHandle;
    if (!h->port) {
        delete h;
        return nullptr;
    }
    elips::gpu::GpuConfig config;
    config.default_ef_search_gpu = nprobe;
    config.ivf_pq_params.n_lists = n_lists;
    config.ivf_pq_params.pq_dim = pq_dim;
    config.ivf_pq_params.pq_bits = pq_bits;
    h->index = std::make_unique<elips::gpu::GpuIVFPQIndex>(*h->port, static_cast<Metric>(metric),
                                                           static_cast<std::uint16_t>(dim), config);
    elips::IndexSnapshot snap;
    snap.kind = elips::IndexSnapshotKind::gpu_ivf_pq;
    snap.metric = static_cast<Metric>(metric);
    snap.dimension = static_cast<std::uint16_t>(dim);
    snap.ids.reserve(n);
    for (size_t i = 0; i < n; ++i) snap.ids.push_back(row_id(i));
    snap.vectors.assign(vectors, vectors + n * dim);
    elips::IvfSnapshot ivf;
    ivf.n_lists = n_lists;
    ivf.n_probe = nprobe;
    ivf.centroids.assign(centroids, centroids + n_lists * dim);
    ivf.assignments.assign(assignments, assignments + n);
    snap.ivf = std::move(ivf);
    elips::PqSnapshot pq;
    pq.pq_dim = pq_dim;
    pq.pq_bits = pq_bits;
    pq.codebook.assign(codebook,
                       codebook + static_cast<size_t>(pq_dim) * (size_t{1} << pq_bits) * (dim / pq_dim));
    pq.codes.assign(codes, codes + n * pq_dim);
    snap.pq = std::move(pq);
    auto imported = h->index->import_snapshot(snap);
    if (!imported.has_value()) {
        delete h;
        return nullptr;
    }
    return h;
}

int ref_ivfpq_search(void* handle, uint32_t dim, const float* queries, size_t nq, size_t k,
                     int nthreads, float* out_dist, std::int64_t* out_rows) {
    auto* h = static_cast<IvfPqHandle*>(handle);
    parallel_queries(nq, nthreads, [&](size_t q) {
        const auto hits = h->index->search(std::span<const float>{queries + q * dim, dim}, k);
        write_hits(hits, k, out_dist + q * k, out_rows + q * k);
    });
    return 0;
}

// GpuIVFPQIndex::remove (state remove, then rebuild_codes), by original row.
int ref_ivfpq_remove(void* handle, size_t row) {
    static_cast<IvfPqHandle*>(handle)->index->remove(row_id(row));
    return 0;
}

// export_snapshot: ids (as original rows), vectors, assignments, codebook, codes.
int ref_ivfpq_export(void* handle, size_t n, uint32_t dim, std::int64_t* rows_out, float* vectors_out,
                     uint32_t* assign_out, float* codebook_out, size_t codebook_len, std::uint8_t* codes_out,
                     size_t codes_len) {
    auto snap = static_cast<IvfPqHandle*>(handle)->index->export_snapshot();
    if (!snap.has_value() || !snap->ivf.has_value() || !snap->pq.has_value()) return 1;
    if (snap->ids.size() != n || snap->vectors.size() != n * dim || snap->ivf->assignments.size() != n) return 2;
    if (snap->pq->codebook.size() != codebook_len || snap->pq->codes.size() != codes_len) return 3;
    for (size_t i = 0; i < n; ++i) rows_out[i] = id_row(snap->ids[i]);
    std::copy(snap->vectors.begin(), snap->vectors.end(), vectors_out);
    std::copy(snap->ivf->assignments.begin(), snap->ivf->assignments.end(), assign_out);
    std::copy(snap->pq->codebook.begin(), snap->pq->codebook.end(), codebook_out);
    std::copy(snap->pq->codes.begin(), snap->pq->codes.end(), codes_out);
    return 0;
}

// export_snapshot's IVF centroids [n_lists][dim]; returns the list count, 0 when untrained.
size_t ref_ivfpq_centroids(void* handle, float* out, size_t cap) {
    auto snap = static_cast<IvfPqHandle*>(handle)->index->export_snapshot();
    if (!snap.has_value() || !snap->ivf.has_value()) return 0;
    std::copy_n(snap->ivf->centroids.begin(), std::min(cap, snap->ivf->centroids.size()), out);
    return snap->ivf->n_lists;
}

void ref_ivfpq_destroy(void* handle) { delete static_cast<IvfPqHandle*>(handle); }

// GpuIVFFlatIndex on the CPU port, loaded through import_snapshot
// (GpuIVFFlatIndex.cpp:202-205, IvfIndexState.cpp:339-374).
void* ref_ivfflat_create(int metric, uint32_t dim, size_t n_lists, size_t nprobe, const float* centroids,
                         const uint32_t* assignments, const float* vectors, size_t n) {
    auto* h = new IvfFlatHandle;
    if (!h->port) {
        delete h;
        return nullptr;
    }
    elips::gpu::GpuConfig config;
    config.default_ef_search_gpu = nprobe;
    config.ivf_pq_params.n_lists = n_lists;
    h->index = std::make_unique<elips::gpu::GpuIVFFlatIndex>(*h->port, static_cast<Metric>(metric),
                                                             static_cast<std::uint16_t>(dim), config);
    elips::IndexSnapshot snap;
    snap.kind = elips::IndexSnapshotKind::gpu_ivf_flat;
    snap.metric = static_cast<Metric>(metric);
    snap.dimension = static_cast<std::uint16_t>(dim);
    snap.ids.reserve(n);
    for (size_t i = 0; i < n; ++i) snap.ids.push_back(row_id(i));
    snap.vectors.assign(vectors, vectors + n * dim);
    elips::IvfSnapshot ivf;
    ivf.n_lists = n_lists;
    ivf.n_probe = nprobe;
    ivf.centroids.assign(centroids, centroids + n_lists * dim);
    ivf.assignments.assign(assignments, assignments + n);
    snap.ivf = std::move(ivf);
    auto imported = h->index->import_snapshot(snap);
    if (!imported.has_value()) {
        delete h;
        return nullptr;
    }
    return h;
}

int ref_ivfflat_search(void* handle, uint32_t dim, const float* queries, size_t nq, size_t k, int nthreads,
                       float* out_dist, std::int64_t* out_rows) {
    auto* h = static_cast<IvfFlatHandle*>(handle);
    parallel_queries(nq, nthreads, [&](size_t q) {
        const auto hits = h->index->search(std::span<const float>{queries + q * dim, dim}, k);
        write_hits(hits, k, out_dist + q * k, out_rows + q * k);
    });
    return 0;
}

// search_batch (GpuIVFFlatIndex.cpp:123-164): batched probe, per-query rank.
int ref_ivfflat_search_batch(void* handle, uint32_t dim, const float* queries, size_t nq, size_t k,
                             float* out_dist, std::int64_t* out_rows) {
    auto* h = static_cast<IvfFlatHandle*>(handle);
    auto res = h->index->search_batch(std::span<const float>{queries, nq * dim}, k, 0);
    if (!res.has_value()) return 1 + static_cast<int>(res.error());
    for (size_t q = 0; q < nq; ++q) {
        const auto& row = (*res)[q];
        for (size_t i = 0; i < k; ++i) {
            if (i < row.size()) {
                out_dist[q * k + i] = row[i].distance;
                out_rows[q * k + i] = id_row(row[i].id);
            } else {
                out_dist[q * k + i] = 0.0f;
                out_rows[q * k + i] = -1;
            }
        }
    }
    return 0;
}

void ref_ivfflat_destroy(void* handle) { delete static_cast<IvfFlatHandle*>(handle); }

// GpuBruteForceIndex (GpuBruteForceIndex.cpp:77-170) over rows with ids
// row_id(i), loaded by build_from_batch (:126-145).
void* ref_brute_create(int metric, uint32_t dim, const float* rows, size_t n) {
    auto* h = new BruteHandle;
    if (!h->port) {
        delete h;
        return nullptr;
    }
    elips::gpu::GpuConfig config;
    h->index = std::make_unique<elips::gpu::GpuBruteForceIndex>(*h->port, static_cast<Metric>(metric),
                                                                static_cast<std::uint16_t>(dim), config);
    std::vector<RecordID> ids;
    ids.reserve(n);
    for (size_t i = 0; i < n; ++i) ids.push_back(row_id(i));
    auto built = h->index->build_from_batch(std::span<const float>{rows, n * dim}, ids, {});
    if (!built.has_value()) {
        delete h;
        return nullptr;
    }
    return h;
}

int ref_brute_search(void* handle, uint32_t dim, const float* queries, size_t nq, size_t k, int nthreads,
                     float* out_dist, std::int64_t* out_rows) {
    auto* h = static_cast<BruteHandle*>(handle);
    parallel_queries(nq, nthreads, [&](size_t q) {
        const auto hits = h->index->search(std::span<const float>{queries + q * dim, dim}, k);
        write_hits(hits, k, out_dist + q * k, out_rows + q * k);
    });
    return 0;
}

// search_batch through GpuSearchPipeline::batch_search (GpuSearchPipeline.cpp:10-41).
int ref_brute_search_batch(void* handle, uint32_t dim, const float* queries, size_t nq, size_t k, float* out_dist,
                           std::int64_t* out_rows) {
    auto* h = static_cast<BruteHandle*>(handle);
    auto res = h->index->search_batch(std::span<const float>{queries, nq * dim}, k, 0);
    if (!res.has_value()) return 1 + static_cast<int>(res.error());
    for (size_t q = 0; q < nq; ++q) {
        const auto& row = (*res)[q];
        for (size_t i = 0; i < k; ++i) {
            out_dist[q * k + i] = i < row.size() ? row[i].distance : 0.0f;
            out_rows[q * k + i] = i < row.size() ? id_row(row[i].id) : -1;
        }
    }
    return 0;
}

void ref_brute_destroy(void* handle) { delete static_cast<BruteHandle*>(handle); }

#ifdef REF_WITH_B200
// ---- the B200 index adapters (elips_b200/integration/B200Indexes.cpp) driven
// through the reference's own interfaces: IndexPort, GpuIndexPort,
// IndexTransferPort, selected by make_b200_index with an elips::Config.

}  // extern "C"

namespace {

struct B200Handle {
    std::unique_ptr<elips::IndexPort> index;
};

elips::gpu::GpuIndexPort* as_gpu(void* h) {
    return dynamic_cast<elips::gpu::GpuIndexPort*>(static_cast<B200Handle*>(h)->index.get());
}

void* wrap(std::unique_ptr<elips::IndexPort> index) {
    if (!index) return nullptr;
    auto* h = new B200Handle;
    h->index = std::move(index);
    return h;
}

}  // namespace

extern "C" {

// make_index's selection (IndexFactory.cpp:40-50) with the B200 classes:
// algorithm 4 = BruteForce, 3 = IvfPq (GpuIndexAlgorithm order); precision
// as GpuPrecision with BF16 = 4.
void* ref_b200_index_create(int metric, uint32_t dim, int algorithm, int precision, size_t n_lists,
                            size_t nprobe, uint32_t pq_dim, uint32_t pq_bits, size_t kmeans_iters) {
    elips::gpu::GpuConfig g;
    g.policy = elips::gpu::GpuPolicy::RequireGpu;
    g.index_build_mode = elips::gpu::IndexBuildMode::GpuBuild_GpuServe;
    g.algorithm = static_cast<elips::gpu::GpuIndexAlgorithm>(algorithm);
    g.search_precision = static_cast<elips::gpu::GpuPrecision>(precision);
    g.default_ef_search_gpu = nprobe;
    g.ivf_pq_params.n_lists = n_lists;
    g.ivf_pq_params.pq_dim = pq_dim;
    g.ivf_pq_params.pq_bits = pq_bits;
    g.ivf_pq_params.kmeans_n_iters = kmeans_iters;
    g.device_index = 0;
    elips::Config config;
    config.metric(static_cast<Metric>(metric)).index(elips::IndexType::exact).gpu(g);
    return wrap(elips::gpu::b200::make_b200_index(config, static_cast<std::uint16_t>(dim)));
}

// A quantized vault's index: make_b200_index with the reference's trained
// quantizer attached (codec 3 = sq8 from mins/scales, 1 = PQ from a codebook,
// 2 = OPQ with a rotation), the CPU twin of ref_sq8/pq/opq_exact_create.
void* ref_b200_quant_index_create(int metric, uint32_t dim, int codec, uint32_t pq_dim, uint32_t pq_bits,
                                  const float* params, const float* rotation) {
    elips::quant::QuantizerPtr q;
    if (codec == 3) {
        q = std::make_shared<elips::quant::ScalarQuantizer>(static_cast<Metric>(metric), static_cast<std::uint16_t>(dim),
                                                            std::vector<float>(params, params + dim),
                                                            std::vector<float>(params + dim, params + 2 * dim));
    } else {
        const size_t cb = static_cast<size_t>(pq_dim) * (size_t{1} << pq_bits) * (dim / pq_dim);
        q = std::make_shared<elips::quant::ProductQuantizer>(
            static_cast<Metric>(metric), static_cast<std::uint16_t>(dim), pq_dim, pq_bits,
            std::vector<float>(params, params + cb),
            codec == 2 ? std::vector<float>(rotation, rotation + static_cast<size_t>(dim) * dim) : std::vector<float>{});
    }
    elips::gpu::GpuConfig g;
    g.policy = elips::gpu::GpuPolicy::RequireGpu;
    g.algorithm = elips::gpu::GpuIndexAlgorithm::BruteForce;
    elips::Config config;
    config.metric(static_cast<Metric>(metric)).index(elips::IndexType::exact).gpu(g);
    config.attach_quantizer(q);
    return wrap(elips::gpu::b200::make_b200_index(config, static_cast<std::uint16_t>(dim)));
}

// IndexPort::insert of rows [first, first + n) with ids row_id(first + i).
// Returns 1 when insert threw DimensionMismatch (width != dim).
int ref_b200_index_insert(void* h, const float* rows, size_t n, size_t width, size_t first) {
    try {
        for (size_t i = 0; i < n; ++i)
            static_cast<B200Handle*>(h)->index->insert(row_id(first + i), std::span<const float>{rows + i * width, width});
    } catch (const elips::DimensionMismatch&) {
        return 1;
    }
    return 0;
}

int ref_b200_index_remove(void* h, size_t row) {
    static_cast<B200Handle*>(h)->index->remove(row_id(row));
    return 0;
}

// GpuIndexPort::build_from_batch with ids row_id(i); 1 + GpuError on failure.
int ref_b200_index_build(void* h, const float* rows, size_t n, uint32_t dim) {
    auto* g = as_gpu(h);
    if (g == nullptr) return -1;
    std::vector<RecordID> ids;
    ids.reserve(n);
    for (size_t i = 0; i < n; ++i) ids.push_back(row_id(i));
    auto r = g->build_from_batch(std::span<const float>{rows, n * dim}, ids, {});
    return r.has_value() ? 0 : 1 + static_cast<int>(r.error());
}

// IndexPort::search per query on nthreads threads (Vault::seek's readers).
// Returns 1 when a query threw DimensionMismatch (width != index dimension).
int ref_b200_index_search(void* h, uint32_t width, const float* queries, size_t nq, size_t k, int nthreads,
                          float* out_dist, std::int64_t* out_rows) {
    std::atomic<int> mismatch{0};
    parallel_queries(nq, nthreads, [&](size_t q) {
        try {
            const auto hits = static_cast<B200Handle*>(h)->index->search(
                std::span<const float>{queries + q * width, width}, k);
            write_hits(hits, k, out_dist + q * k, out_rows + q * k);
        } catch (const elips::DimensionMismatch&) {
            mismatch = 1;
        }
    });
    return mismatch.load();
}

// GpuIndexPort::search_batch; 1 + GpuError on failure. With candidates
// (n_cand > 0 or candidates != NULL) the brute-force index's filtered search
// over ids row_id(candidates[i]).
int ref_b200_index_search_batch(void* h, uint32_t dim, const float* queries, size_t nq, size_t k,
                                const std::int64_t* candidates, size_t n_cand, float* out_dist,
                                std::int64_t* out_rows) {
    auto* g = as_gpu(h);
    if (g == nullptr) return -1;
    std::expected<std::vector<std::vector<elips::SearchResult>>, elips::gpu::GpuError> res;
    if (candidates != nullptr) {
        auto* bf = dynamic_cast<elips::gpu::b200::B200BruteForceIndex*>(g);
        if (bf == nullptr) return -2;
        std::vector<RecordID> ids;
        for (size_t i = 0; i < n_cand; ++i) ids.push_back(row_id(static_cast<std::uint64_t>(candidates[i])));
        res = bf->search_batch_filtered(std::span<const float>{queries, nq * dim}, k, ids);
    } else {
        res = g->search_batch(std::span<const float>{queries, nq * dim}, k, 0);
    }
    if (!res.has_value()) return 1 + static_cast<int>(res.error());
    for (size_t q = 0; q < nq; ++q) {
        const auto& row = (*res)[q];
        for (size_t i = 0; i < k; ++i) {
            out_dist[q * k + i] = i < row.size() ? row[i].distance : 0.0f;
            out_rows[q * k + i] = i < row.size() ? id_row(row[i].id) : -1;
        }
    }
    return 0;
}

size_t ref_b200_index_size(void* h) { return static_cast<B200Handle*>(h)->index->size(); }

// type_name() into buf (NUL-terminated, truncated to cap).
void ref_b200_index_type_name(void* h, char* buf, size_t cap) {
    const auto name = static_cast<B200Handle*>(h)->index->type_name();
    const size_t n = std::min(cap - 1, name.size());
    std::memcpy(buf, name.data(), n);
    buf[n] = 0;
}

size_t ref_b200_index_device_bytes(void* h) {
    auto* g = as_gpu(h);
    return g != nullptr ? g->device_bytes_used() : 0;
}

// export_snapshot of src imported into dst (IndexTransferPort); 0 on success.
int ref_b200_index_snapshot_copy(void* src, void* dst) {
    auto* s = dynamic_cast<elips::IndexTransferPort*>(static_cast<B200Handle*>(src)->index.get());
    auto* d = dynamic_cast<elips::IndexTransferPort*>(static_cast<B200Handle*>(dst)->index.get());
    if (s == nullptr || d == nullptr) return 1;
    auto snap = s->export_snapshot();
    if (!snap.has_value()) return 2;
    return d->import_snapshot(*snap).has_value() ? 0 : 3;
}

// GpuIndexPort::export_to_cpu_index into a new CPU ExactIndex (an ExactHandle
// searched with ref_exact_search), or import_from_cpu_index from one (dir = 1).
void* ref_b200_index_export_to_cpu(void* h, int metric, uint32_t dim) {
    auto* g = as_gpu(h);
    if (g == nullptr) return nullptr;
    auto* e = new ExactHandle;
    e->index = std::make_unique<elips::ExactIndex>(static_cast<Metric>(metric), static_cast<std::uint16_t>(dim));
    if (!g->export_to_cpu_index(*e->index).has_value()) {
        delete e;
        return nullptr;
    }
    return e;
}

int ref_b200_index_import_from_cpu(void* h, void* exact_handle) {
    auto* g = as_gpu(h);
    if (g == nullptr) return -1;
    auto r = g->import_from_cpu_index(*static_cast<ExactHandle*>(exact_handle)->index);
    return r.has_value() ? 0 : 1 + static_cast<int>(r.error());
}

// export_snapshot's IVF-PQ fields (as ref_ivfpq_export): ids as rows, vectors,
// assignments, codebook, codes. 1..3 when a section is missing or mis-sized.
int ref_b200_index_export(void* h, size_t n, uint32_t dim, std::int64_t* rows_out, float* vectors_out,
                          uint32_t* assign_out, float* codebook_out, size_t codebook_len, std::uint8_t* codes_out,
                          size_t codes_len) {
    auto* t = dynamic_cast<elips::IndexTransferPort*>(static_cast<B200Handle*>(h)->index.get());
    if (t == nullptr) return 4;
    auto snap = t->export_snapshot();
    if (!snap.has_value() || !snap->ivf.has_value() || !snap->pq.has_value()) return 1;
    if (snap->ids.size() != n || snap->vectors.size() != n * dim || snap->ivf->assignments.size() != n) return 2;
    if (snap->pq->codebook.size() != codebook_len || snap->pq->codes.size() != codes_len) return 3;
    for (size_t i = 0; i < n; ++i) rows_out[i] = id_row(snap->ids[i]);
    std::copy(snap->vectors.begin(), snap->vectors.end(), vectors_out);
    std::copy(snap->ivf->assignments.begin(), snap->ivf->assignments.end(), assign_out);
    std::copy(snap->pq->codebook.begin(), snap->pq->codebook.end(), codebook_out);
    std::copy(snap->pq->codes.begin(), snap->pq->codes.end(), codes_out);
    return 0;
}

size_t ref_b200_index_centroids(void* h, float* out, size_t cap) {
    auto* t = dynamic_cast<elips::IndexTransferPort*>(static_cast<B200Handle*>(h)->index.get());
    if (t == nullptr) return 0;
    auto snap = t->export_snapshot();
    if (!snap.has_value() || !snap->ivf.has_value()) return 0;
    std::copy_n(snap->ivf->centroids.begin(), std::min(cap, snap->ivf->centroids.size()), out);
    return snap->ivf->n_lists;
}

void ref_b200_index_destroy(void* h) { delete static_cast<B200Handle*>(h); }
#endif  // REF_WITH_B200

// CPU counterparts for the insert / remove sequences: ExactIndex::insert /
// remove, and GpuIVFPQIndex built empty then filled by insert or
// build_from_batch (on the CPU port).
int ref_exact_insert(void* handle, const float* rows, size_t n, uint32_t dim, size_t first) {
    auto* h = static_cast<ExactHandle*>(handle);
    for (size_t i = 0; i < n; ++i) h->index->insert(row_id(first + i), std::span<const float>{rows + i * dim, dim});
    return 0;
}

int ref_exact_remove(void* handle, size_t row) {
    static_cast<ExactHandle*>(handle)->index->remove(row_id(row));
    return 0;
}

size_t ref_exact_size(void* handle) { return static_cast<ExactHandle*>(handle)->index->size(); }

void* ref_ivfpq_create_empty(int metric, uint32_t dim, size_t n_lists, size_t nprobe, uint32_t pq_dim,
                             uint32_t pq_bits, size_t kmeans_iters) {
    auto* h = new IvfPqHandle;
    if (!h->port) {
        delete h;
        return nullptr;
    }
    elips::gpu::GpuConfig config;
    config.default_ef_search_gpu = nprobe;
    config.ivf_pq_params.n_lists = n_lists;
    config.ivf_pq_params.pq_dim = pq_dim;
    config.ivf_pq_params.pq_bits = pq_bits;
    config.ivf_pq_params.kmeans_n_iters = kmeans_iters;
    h->index = std::make_unique<elips::gpu::GpuIVFPQIndex>(*h->port, static_cast<Metric>(metric),
                                                           static_cast<std::uint16_t>(dim), config);
    return h;
}

int ref_ivfpq_insert(void* handle, const float* rows, size_t n, uint32_t dim, size_t first) {
    auto* h = static_cast<IvfPqHandle*>(handle);
    for (size_t i = 0; i < n; ++i) h->index->insert(row_id(first + i), std::span<const float>{rows + i * dim, dim});
    return 0;
}

int ref_ivfpq_build(void* handle, const float* rows, size_t n, uint32_t dim) {
    auto* h = static_cast<IvfPqHandle*>(handle);
    std::vector<RecordID> ids;
    for (size_t i = 0; i < n; ++i) ids.push_back(row_id(i));
    return h->index->build_from_batch(std::span<const float>{rows, n * dim}, ids, {}).has_value() ? 0 : 1;
}

size_t ref_ivfpq_size(void* handle) { return static_cast<IvfPqHandle*>(handle)->index->size(); }

// Selects the GpuPort of the handles created next: 1 = the B200 CudaBackend
// (REF_WITH_B200 build only), 0 = the CPU port. Returns the selection made.
int ref_use_b200_port(int on) {
#ifdef REF_WITH_B200
    g_use_b200.store(on ? 1 : 0);
    return on ? 1 : 0;
#else
    (void)on;
    return 0;
#endif
}

}  // extern "C"
