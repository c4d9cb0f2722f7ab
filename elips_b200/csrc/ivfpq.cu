// Host side of the IVF indexes: GpuIVFPQIndex (src/gpu_engine/
// GpuIVFPQIndex.cpp) and GpuIVFFlatIndex (src/gpu_engine/GpuIVFFlatIndex.cpp)
// with their model (centroids, list assignments, and for IVF-PQ the residual
// codebook and codes) imported as import_snapshot does (GpuIVFPQIndex.cpp:
// 327-348, IvfIndexState.cpp:339-374), rows resident on the device, per-list
// data stored list-major.
#include <algorithm>
#include <cstdio>
#include <vector>

#include "../../include/elips_b200.h"
#include "engine.cuh"
#include "capi_util.cuh"
#include "train.cuh"
#include "ivfpq_kernels.cuh"
#include "profiler.cuh"

namespace eb {

void compute_distances_device(int device, const float* q, const float* db, float* out, size_t nq, size_t nb,
                              size_t d, int metric, cudaStream_t stream);
void top_k_device(int device, const float* dist, uint32_t* idx, float* val, size_t nq, size_t nb, size_t k,
                  cudaStream_t stream);

namespace {

size_t a256(size_t x) { return (x + 255) / 256 * 256; }

void launch_ok(const char* what) { check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, what); }

}  // namespace

// Rows, list assignments and inverted lists shared by the IVF indexes
// (detail::IvfIndexState), plus the probe and the probe plan of a search.
class IvfLists {
public:
    IvfLists(int device, int metric, uint32_t dim, uint32_t nlist, uint32_t nprobe, const float* centroids)
        : device_(device), metric_(metric), dim_(dim), nlist_(nlist), nprobe_(std::max<uint32_t>(1, nprobe)),
          owned_host_(nlist, true), members_(nlist) {
        if (metric < 0 || metric > 2) fail(ELIPS_B200_UNSUPPORTED_METRIC, "unknown metric");
        if (dim == 0 || dim > 65535 || nlist == 0) fail(ELIPS_B200_INVALID_ARGUMENT, "bad dimension or list count");
        if (centroids == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "centroids are null");
        device_props(device);
        DeviceGuard g(device);
        centroids_ = DeviceBuffer(device, static_cast<size_t>(nlist) * dim * 4);
        check_cuda(cudaMemcpy(centroids_.get(), centroids, static_cast<size_t>(nlist) * dim * 4, cudaMemcpyHostToDevice),
                   ELIPS_B200_TRANSFER_FAILED, "centroids");
    }

    int device() const { return device_; }
    uint32_t dim() const { return dim_; }
    size_t size() const { return n_; }
    void set_nprobe(uint32_t nprobe) { nprobe_ = std::max<uint32_t>(1, nprobe); }

    // The lists this index owns as one GPU's share of a list-sharded index
    // (GpuDistributedIndex over IVF lists): bit l & 31 of words[l >> 5]
    // (ceil(n_lists / 32) words, HOST). Rows may only name owned lists, and a
    // search scans only them. Default: every list.
    void set_owned_lists(const uint32_t* words, size_t n_words) {
        if (words == nullptr || n_words != (nlist_ + 31u) / 32u)
            fail(ELIPS_B200_INVALID_ARGUMENT, "owned-list mask must have ceil(n_lists / 32) words");
        std::vector<bool> owned(nlist_);
        for (uint32_t l = 0; l < nlist_; ++l) owned[l] = (words[l >> 5] >> (l & 31u)) & 1u;
        for (uint32_t a : assign_)
            if (!owned[a]) fail(ELIPS_B200_INVALID_ARGUMENT, "rows already added on a list outside the mask");
        DeviceGuard g(device_);
        owned_ = DeviceBuffer(device_, n_words * 4);
        check_cuda(cudaMemcpy(owned_.get(), words, n_words * 4, cudaMemcpyHostToDevice), ELIPS_B200_TRANSFER_FAILED,
                   "owned lists");
        owned_host_ = std::move(owned);
    }

    // Lists [lo, hi) only (a contiguous share).
    void set_list_range(uint32_t lo, uint32_t hi) {
        if (lo > hi || hi > nlist_) fail(ELIPS_B200_INVALID_ARGUMENT, "list range outside [0, n_lists]");
        std::vector<uint32_t> words((nlist_ + 31u) / 32u, 0u);
        for (uint32_t l = lo; l < hi; ++l) words[l >> 5] |= 1u << (l & 31u);
        set_owned_lists(words.data(), words.size());
    }

    // IvfIndexState::remove (IvfIndexState.cpp:262-326) on the device: the
    // slot leaves its list; unless it is the last slot, the last slot's row
    // (vector, list, derived data) moves into it and keeps its place in its
    // list under the new number; the store shrinks by one. No re-upload: one
    // row copied on the device, the lists rebuilt from the member order at
    // the next search. (The reference also retrains when fewer rows than
    // lists remain; that case is the caller's: train again and re-add.)
    void remove(size_t slot, cudaStream_t stream) {
        if (slot >= n_) fail(ELIPS_B200_INVALID_ARGUMENT, "slot out of range");
        DeviceGuard g(device_);
        const size_t last = n_ - 1;
        auto& mine = members_[assign_[slot]];
        mine.erase(std::find(mine.begin(), mine.end(), static_cast<uint32_t>(slot)));
        if (slot != last) {
            float* v = static_cast<float*>(vectors_.get());
            check_cuda(cudaMemcpyAsync(v + slot * dim_, v + last * dim_, static_cast<size_t>(dim_) * 4,
                                       cudaMemcpyDeviceToDevice, stream),
                       ELIPS_B200_TRANSFER_FAILED, "row move");
            move_row(last, slot, stream);
            assign_[slot] = assign_[last];
            auto& moved = members_[assign_[slot]];
            *std::find(moved.begin(), moved.end(), static_cast<uint32_t>(last)) = static_cast<uint32_t>(slot);
        }
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "remove");
        assign_.pop_back();
        --n_;
        dirty_ = true;
    }

protected:
    // Validates the list ids (they must name a list), grows the row store and
    // appends the rows (DEVICE pointers). Returns the host copy of the ids;
    // the caller appends its own per-row data, then calls commit_rows.
    std::vector<uint32_t> append_rows(const float* vectors, const uint32_t* assign, size_t n, cudaStream_t stream) {
        if (vectors == nullptr || assign == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "vectors and assignments are required");
        if (n_ + n >= 0xFFFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "index limited to 2^32-2 rows");
        std::vector<uint32_t> host_assign(n);
        check_cuda(cudaMemcpyAsync(host_assign.data(), assign, n * 4, cudaMemcpyDeviceToHost, stream),
                   ELIPS_B200_TRANSFER_FAILED, "assignment copy");
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_TRANSFER_FAILED, "assignment copy");
        for (uint32_t a : host_assign) {
            if (a >= nlist_) fail(ELIPS_B200_INVALID_ARGUMENT, "assignment names a list past n_lists");
            if (!owned_host_[a]) fail(ELIPS_B200_INVALID_ARGUMENT, "assignment names a list this index does not own");
        }
        if (n_ + n > capacity_) {
            const size_t cap = std::max<size_t>(n_ + n, capacity_ + capacity_ / 2);
            DeviceBuffer v(device_, cap * dim_ * 4);
            if (n_ > 0)
                check_cuda(cudaMemcpy(v.get(), vectors_.get(), n_ * dim_ * 4, cudaMemcpyDeviceToDevice),
                           ELIPS_B200_TRANSFER_FAILED, "grow copy");
            vectors_ = std::move(v);
            capacity_ = cap;
            grow(cap);
        }
        check_cuda(cudaMemcpyAsync(static_cast<float*>(vectors_.get()) + n_ * dim_, vectors, n * dim_ * 4,
                                   cudaMemcpyDeviceToDevice, stream),
                   ELIPS_B200_TRANSFER_FAILED, "vector copy");
        return host_assign;
    }

    void commit_rows(const std::vector<uint32_t>& host_assign, cudaStream_t stream) {
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "ivf add");
        for (size_t i = 0; i < host_assign.size(); ++i) members_[host_assign[i]].push_back(static_cast<uint32_t>(n_ + i));
        assign_.insert(assign_.end(), host_assign.begin(), host_assign.end());
        n_ += host_assign.size();
        dirty_ = true;
    }

    // Derived stores grow their per-row data to `rows` (existing rows kept).
    virtual void grow(size_t rows) = 0;
    // Derived stores rebuild their list-major copies after the lists change.
    virtual void gather_lists(cudaStream_t stream) = 0;
    // Derived stores move one row's data from slot `from` to slot `to`.
    virtual void move_row(size_t from, size_t to, cudaStream_t stream) = 0;

    // Lists in member order: ascending slots as rows are added
    // (IvfIndexState::rebuild_list_members, IvfIndexState.cpp:75-83), a moved
    // row keeping its place after a remove (IvfIndexState.cpp:285-301); then
    // the derived list-major copies.
    void finalize(cudaStream_t stream) {
        if (!dirty_) return;
        std::vector<uint32_t> off(nlist_ + 1, 0);
        for (uint32_t l = 0; l < nlist_; ++l) off[l + 1] = off[l] + static_cast<uint32_t>(members_[l].size());
        std::vector<uint32_t> rows(n_);
        for (uint32_t l = 0; l < nlist_; ++l) std::copy(members_[l].begin(), members_[l].end(), rows.begin() + off[l]);
        list_off_ = DeviceBuffer(device_, off.size() * 4);
        list_rows_ = DeviceBuffer(device_, std::max<size_t>(n_, 1) * 4);
        check_cuda(cudaMemcpyAsync(list_off_.get(), off.data(), off.size() * 4, cudaMemcpyHostToDevice, stream),
                   ELIPS_B200_TRANSFER_FAILED, "list offsets");
        check_cuda(cudaMemcpyAsync(list_rows_.get(), rows.data(), n_ * 4, cudaMemcpyHostToDevice, stream),
                   ELIPS_B200_TRANSFER_FAILED, "list rows");
        gather_lists(stream);
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "list build");
        dirty_ = false;
    }

    struct Plan {
        uint32_t* probes = nullptr;
        uint32_t* counts = nullptr;
        uint32_t* list_start = nullptr;
        uint32_t* pairs = nullptr;
        uint2* items = nullptr;
        uint32_t* ctrl = nullptr;
        uint32_t* qbound = nullptr;
        uint32_t* pair_off = nullptr;
        uint2* part = nullptr;
        size_t npairs = 0;
        uint32_t nprobe = 0;
    };

    // Scratch bytes of a plan for nq queries keeping r candidates per pair.
    size_t plan_bytes(size_t nq, uint32_t r, bool flat) const {
        const uint32_t nprobe = std::min(nprobe_, nlist_);
        const size_t npairs = nq * nprobe;
        return a256(nq * nlist_ * 4) + 2 * a256(npairs * 4) + a256(npairs * static_cast<size_t>(r) * 8) +
               3 * a256(static_cast<size_t>(nlist_) * 4) + a256(npairs * 4) + a256((npairs + nlist_) * 8) + 256 +
               a256(nq * 4) + (flat ? a256(npairs * 4) : 0);
    }

    // Probe (IvfIndexState::probe_lists, IvfIndexState.cpp:395-423: exact
    // distances to the centroids, then the nprobe best) and group the
    // (query, probe) pairs by list for G queries per scan item. Carves its
    // scratch from w.
public:
    // The nprobe nearest lists of every query (IvfIndexState::probe_lists,
    // IvfIndexState.cpp:395-464): exact distances to every centroid, then the
    // nprobe smallest, ties by list id. probes: [nq][nprobe] DEVICE.
    void probe(const float* queries, size_t nq, uint32_t* probes, cudaStream_t stream) const {
        if (nq == 0) return;
        if (queries == nullptr || probes == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "null pointer");
        DeviceGuard g(device_);
        const uint32_t nprobe = std::min(nprobe_, nlist_);
        StreamScratch s(a256(nq * nlist_ * 4) + a256(nq * nprobe * 4), stream);
        float* dist = reinterpret_cast<float*>(s.get());
        float* pval = reinterpret_cast<float*>(s.get() + a256(nq * nlist_ * 4));
        compute_distances_device(device_, queries, static_cast<const float*>(centroids_.get()), dist, nq, nlist_, dim_,
                                 metric_, stream);
        top_k_device(device_, dist, probes, pval, nq, nlist_, nprobe, stream);
    }

    uint32_t probes_per_query() const { return std::min(nprobe_, nlist_); }

protected:

    // probes_in (optional, DEVICE [nq][nprobe]): probe lists computed
    // elsewhere (another rank's slice of the batch), used instead of probing.
    // shared_bound (optional, DEVICE [nq], possibly another GPU's memory):
    // per-query admission bounds shared with other shards searching the same
    // batch, used instead of this search's own (and not reset here).
    Plan probe_and_plan(const float* queries, size_t nq, uint32_t r, uint32_t G, bool flat, uint8_t*& w,
                        cudaStream_t stream, const uint32_t* probes_in = nullptr,
                        uint32_t* shared_bound = nullptr) {
        Plan pl;
        pl.nprobe = std::min(nprobe_, nlist_);
        pl.npairs = nq * pl.nprobe;
        auto carve = [&](size_t bytes) {
            uint8_t* at = w;
            w += bytes;
            return at;
        };
        float* dist = reinterpret_cast<float*>(carve(a256(nq * nlist_ * 4)));
        pl.probes = reinterpret_cast<uint32_t*>(carve(a256(pl.npairs * 4)));
        float* pval = reinterpret_cast<float*>(carve(a256(pl.npairs * 4)));
        pl.part = reinterpret_cast<uint2*>(carve(a256(pl.npairs * static_cast<size_t>(r) * 8)));
        pl.counts = reinterpret_cast<uint32_t*>(carve(a256(static_cast<size_t>(nlist_) * 4)));
        pl.list_start = reinterpret_cast<uint32_t*>(carve(a256(static_cast<size_t>(nlist_) * 4)));
        uint32_t* cursor = reinterpret_cast<uint32_t*>(carve(a256(static_cast<size_t>(nlist_) * 4)));
        pl.pairs = reinterpret_cast<uint32_t*>(carve(a256(pl.npairs * 4)));
        pl.items = reinterpret_cast<uint2*>(carve(a256((pl.npairs + nlist_) * 8)));
        pl.ctrl = reinterpret_cast<uint32_t*>(carve(256));
        pl.qbound = reinterpret_cast<uint32_t*>(carve(a256(nq * 4)));
        if (flat) pl.pair_off = reinterpret_cast<uint32_t*>(carve(a256(pl.npairs * 4)));
        if (probes_in != nullptr) {
            check_cuda(cudaMemcpyAsync(pl.probes, probes_in, pl.npairs * 4, cudaMemcpyDeviceToDevice, stream),
                       ELIPS_B200_TRANSFER_FAILED, "probe copy");
        } else {
            compute_distances_device(device_, queries, static_cast<const float*>(centroids_.get()), dist, nq, nlist_,
                                     dim_, metric_, stream);
            top_k_device(device_, dist, pl.probes, pval, nq, nlist_, pl.nprobe, stream);
        }
        check_cuda(cudaMemsetAsync(pl.counts, 0, static_cast<size_t>(nlist_) * 4, stream),
                   ELIPS_B200_KERNEL_LAUNCH_FAILED, "pair counts");
        if (shared_bound != nullptr) pl.qbound = shared_bound;
        else
            check_cuda(cudaMemsetAsync(pl.qbound, 0xFF, nq * 4, stream), ELIPS_B200_KERNEL_LAUNCH_FAILED,
                       "query bounds");
        const uint32_t pblocks = static_cast<uint32_t>((pl.npairs + 255) / 256);
        const uint32_t* loff = static_cast<const uint32_t*>(list_off_.get());
        {
            Profiler::Scope prof("ivfpq_plan", stream, pl.npairs);
            ivf_pair_count_kernel<<<pblocks, 256, 0, stream>>>(pl.probes, static_cast<uint32_t>(pl.npairs), nlist_,
                                                               owned_words(), pl.counts, pl.part, r);
            launch_ok("pair count kernel");
        }
        {
            uint32_t npow2 = 1;
            while (npow2 < nlist_) npow2 <<= 1;
            const size_t psmem = nlist_ <= kPlanSortMax ? static_cast<size_t>(npow2) * 8 : 0;
            allow_dynamic_smem(reinterpret_cast<const void*>(ivf_group_plan_kernel), psmem);
            Profiler::Scope prof("ivfpq_plan", stream, nlist_);
            ivf_group_plan_kernel<<<1, kPlanThreads, psmem, stream>>>(pl.counts, loff, nlist_, G, pl.list_start,
                                                                      cursor, pl.items, pl.ctrl);
            launch_ok("group plan kernel");
        }
        {
            Profiler::Scope prof("ivfpq_plan", stream, pl.npairs);
            ivf_pair_scatter_kernel<<<pblocks, 256, 0, stream>>>(pl.probes, static_cast<uint32_t>(pl.npairs), nlist_,
                                                                 owned_words(), pl.list_start, cursor, pl.pairs);
            launch_ok("pair scatter kernel");
        }
        if (flat) {
            Profiler::Scope prof("ivfpq_plan", stream, nq);
            ivf_pair_offsets_kernel<<<static_cast<uint32_t>((nq + 255) / 256), 256, 0, stream>>>(
                pl.probes, static_cast<uint32_t>(nq), pl.nprobe, nlist_, loff, pl.pair_off);
            launch_ok("pair offsets kernel");
        }
        return pl;
    }

    IvfGroupParams group_params(const float* queries, const Plan& pl, uint32_t r, uint32_t capq,
                                uint32_t lut_stride) const {
        IvfGroupParams p{};
        p.queries = queries;
        p.centroids = static_cast<const float*>(centroids_.get());
        p.list_rows = static_cast<const uint32_t*>(list_rows_.get());
        p.list_off = static_cast<const uint32_t*>(list_off_.get());
        p.counts = pl.counts;
        p.list_start = pl.list_start;
        p.pairs = pl.pairs;
        p.items = pl.items;
        p.ctrl = pl.ctrl;
        p.partial = pl.part;
        p.qbound = pl.qbound;
        p.pair_off = pl.pair_off;
        p.d = dim_;
        p.nprobe = pl.nprobe;
        p.r = r;
        p.capq = capq;
        p.lut_stride = lut_stride;
        p.metric = metric_;
        return p;
    }

    // Queries per scan group: about as many as share a probed list on
    // average, at most 8, and no more than shared memory holds.
    uint32_t group_size(size_t npairs, uint32_t r, uint32_t lut_stride) const {
        const double share = static_cast<double>(npairs) / static_cast<double>(std::min<size_t>(nlist_, npairs));
        uint32_t G = 1;
        while (G < 8 && 2.0 * G <= share) G <<= 1;
        const size_t optin = device_props(device_).max_smem_optin;
        while (G > 1 && group_layout(G, dim_, lut_stride, group_capacity(G, r)).total > optin) G >>= 1;
        return G;
    }

    template <int G, int MB, int BITS, bool FLAT>
    void launch_group(const IvfGroupParams& p, size_t smem, uint64_t max_items, cudaStream_t stream) {
        const auto& props = device_props(device_);
        if (smem > props.max_smem_optin) fail(ELIPS_B200_INVALID_ARGUMENT, "ivf scan needs too much shared memory");
        auto kern = ivfpq_group_scan_kernel<G, MB, BITS, FLAT>;
        allow_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
        int per_sm = 0;
        check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGroupThreads, smem),
                   ELIPS_B200_KERNEL_LAUNCH_FAILED, "occupancy");
        if (per_sm < 1) fail(ELIPS_B200_INVALID_ARGUMENT, "ivf scan does not fit on an SM");
        const uint64_t grid = std::max<uint64_t>(1, std::min<uint64_t>(static_cast<uint64_t>(props.num_sms) * per_sm,
                                                                       max_items));
        Profiler::Scope prof(FLAT ? "ivfflat_scan" : "ivfpq_scan", stream, max_items);
        kern<<<static_cast<uint32_t>(grid), kGroupThreads, smem, stream>>>(p);
        launch_ok("ivf group scan kernel");
    }

public:
    // IndexSnapshot's IVF section and vectors (IndexSnapshot.hpp:26-56) in
    // slot order, into host memory; any output may be null.
    void export_ivf(float* centroids, uint32_t* assignments, float* vectors) const {
        DeviceGuard g(device_);
        check_cuda(cudaDeviceSynchronize(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "export sync");
        if (centroids != nullptr)
            check_cuda(cudaMemcpy(centroids, centroids_.get(), static_cast<size_t>(nlist_) * dim_ * 4,
                                  cudaMemcpyDeviceToHost),
                       ELIPS_B200_TRANSFER_FAILED, "centroid export");
        if (assignments != nullptr) std::copy(assign_.begin(), assign_.end(), assignments);
        if (vectors != nullptr && n_ > 0)
            check_cuda(cudaMemcpy(vectors, vectors_.get(), n_ * dim_ * 4, cudaMemcpyDeviceToHost),
                       ELIPS_B200_TRANSFER_FAILED, "vector export");
    }

protected:
    int device_, metric_;
    uint32_t dim_, nlist_, nprobe_;
    std::vector<bool> owned_host_;
    DeviceBuffer owned_;  // empty: every list

    const uint32_t* owned_words() const { return static_cast<const uint32_t*>(owned_.get()); }
    size_t n_ = 0, capacity_ = 0;
    bool dirty_ = false;
    std::vector<uint32_t> assign_;
    std::vector<std::vector<uint32_t>> members_;  // slots of each list, in list order
    DeviceBuffer centroids_, vectors_, list_off_, list_rows_;
};

class IvfPqIndex : public IvfLists {
public:
    IvfPqIndex(int device, int metric, uint32_t dim, uint32_t nlist, uint32_t nprobe, uint32_t pq_dim,
               uint32_t pq_bits, const float* centroids, const float* codebook)
        : IvfLists(device, metric, dim, nlist, nprobe, centroids), m_(pq_dim) {
        if (pq_dim == 0 || dim % pq_dim != 0 || pq_bits < 4 || pq_bits > 8)
            fail(ELIPS_B200_INVALID_ARGUMENT, "pq_dim must divide the dimension and pq_bits be in [4, 8]");
        if (codebook == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "codebook is null");
        DeviceGuard g(device);
        ksub_ = 1u << pq_bits;
        pq_bits_ = pq_bits;
        if (group_layout(1, dim, group_lut_stride(m_, ksub_), group_capacity(1, 4 * 256)).total >
            device_props(device).max_smem_optin)
            fail(ELIPS_B200_INVALID_ARGUMENT, "pq_dim x 2^pq_bits lookup table too large for shared memory");
        const size_t cb = static_cast<size_t>(m_) * ksub_ * (dim / m_);
        codebook_ = DeviceBuffer(device, cb * 4);
        check_cuda(cudaMemcpy(codebook_.get(), codebook, cb * 4, cudaMemcpyHostToDevice), ELIPS_B200_TRANSFER_FAILED,
                   "codebook");
    }

    uint32_t pq_dim() const { return m_; }

    // GpuIVFPQIndex::rebuild_codes (GpuIVFPQIndex.cpp:88-131), which the
    // reference runs after every insert and remove: the PQ codebook trained
    // again on every row's residual (10 rounds), then every row re-encoded,
    // bit-identical to the CPU code.
    void rebuild_codes(cudaStream_t stream) {
        if (n_ == 0) return;
        DeviceGuard g(device_);
        StreamScratch s(a256(n_ * 4) + n_ * dim_ * 4, stream);
        uint32_t* da = reinterpret_cast<uint32_t*>(s.get());
        float* res = reinterpret_cast<float*>(s.get() + a256(n_ * 4));
        check_cuda(cudaMemcpyAsync(da, assign_.data(), n_ * 4, cudaMemcpyHostToDevice, stream),
                   ELIPS_B200_TRANSFER_FAILED, "assignment upload");
        const uint64_t total = static_cast<uint64_t>(n_) * dim_;
        {
            Profiler::Scope prof("residuals", stream, n_);
            residuals_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(
                static_cast<const float*>(vectors_.get()), da, static_cast<const float*>(centroids_.get()), n_, dim_, res);
            launch_ok("residual kernel");
        }
        train_pq_codebook_device(device_, res, n_, dim_, m_, ksub_, 10, static_cast<float*>(codebook_.get()), stream);
        pq_encode_device(res, n_, dim_, m_, ksub_, static_cast<const float*>(codebook_.get()),
                         static_cast<uint8_t*>(codes_.get()), stream);
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "rebuild codes");
        dirty_ = true;
    }

    // The PQ section of IndexSnapshot: codebook [pq_dim][ksub][dim/pq_dim] and
    // codes [n][pq_dim] in slot order, into host memory; either may be null.
    void export_pq(float* codebook, uint8_t* codes) const {
        DeviceGuard g(device_);
        check_cuda(cudaDeviceSynchronize(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "export sync");
        if (codebook != nullptr)
            check_cuda(cudaMemcpy(codebook, codebook_.get(), static_cast<size_t>(ksub_) * dim_ * 4, cudaMemcpyDeviceToHost),
                       ELIPS_B200_TRANSFER_FAILED, "codebook export");
        if (codes != nullptr && n_ > 0)
            check_cuda(cudaMemcpy(codes, codes_.get(), n_ * m_, cudaMemcpyDeviceToHost), ELIPS_B200_TRANSFER_FAILED,
                       "code export");
    }

    // Appends n rows (DEVICE pointers). assign: list of each row; codes may be
    // null, in which case the residuals are encoded on the device exactly as
    // rebuild_codes does (fp32 x - centroid, then encode_pq).
    void add_device(const float* vectors, const uint32_t* assign, const uint8_t* codes, size_t n, cudaStream_t stream) {
        if (n == 0) return;
        DeviceGuard g(device_);
        const std::vector<uint32_t> host_assign = append_rows(vectors, assign, n, stream);
        uint8_t* cdst = static_cast<uint8_t*>(codes_.get()) + n_ * m_;
        if (codes != nullptr) {
            check_cuda(cudaMemcpyAsync(cdst, codes, n * m_, cudaMemcpyDeviceToDevice, stream), ELIPS_B200_TRANSFER_FAILED,
                       "code copy");
        } else {
            StreamScratch res(n * dim_ * 4, stream);
            const uint64_t total = static_cast<uint64_t>(n) * dim_;
            {
                Profiler::Scope prof("residuals", stream, n);
                residuals_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(
                    vectors, assign, static_cast<const float*>(centroids_.get()), n, dim_,
                    reinterpret_cast<float*>(res.get()));
                launch_ok("residual kernel");
            }
            pq_encode_device(reinterpret_cast<const float*>(res.get()), n, dim_, m_, ksub_,
                             static_cast<const float*>(codebook_.get()), cdst, stream);
        }
        commit_rows(host_assign, stream);
    }

    // Codes of every row in slot order (DEVICE destination, n x pq_dim).
    void read_codes(uint8_t* dst, cudaStream_t stream) const {
        DeviceGuard g(device_);
        if (n_ == 0) return;
        check_cuda(cudaMemcpyAsync(dst, codes_.get(), n_ * m_, cudaMemcpyDeviceToDevice, stream),
                   ELIPS_B200_TRANSFER_FAILED, "code read");
    }

    void search_device(const float* queries, size_t nq, size_t k, float* out_dist, int64_t* out_rows,
                       cudaStream_t stream) {
        if (nq == 0 || k == 0) return;
        check_search(queries, nq, k);
        DeviceGuard g(device_);
        if (n_ == 0) {
            merge_candidates(device_, nullptr, static_cast<uint32_t>(nq), 0, static_cast<uint32_t>(k), 0, 0, 0, out_dist,
                             out_rows, nullptr, stream);
            return;
        }
        const uint32_t r = static_cast<uint32_t>(4 * k);
        StreamScratch s(a256(nq * static_cast<size_t>(r) * 8), stream);
        uint2* cand = reinterpret_cast<uint2*>(s.get());
        candidates(queries, nq, k, cand, stream);
        rerank(queries, nq, k, cand, out_dist, out_rows, stream);
    }

    // Steps 1-4 of search: the R = 4k best (approximate key, slot) per query
    // over the probed lists this index owns, ascending, padded with
    // {+inf, 0xFFFFFFFF}. out_cand: [nq][R] DEVICE.
    void candidates(const float* queries, size_t nq, size_t k, uint2* out_cand, cudaStream_t stream,
                    const uint32_t* probes_in = nullptr, uint32_t* shared_bound = nullptr) {
        if (nq == 0 || k == 0) return;
        check_search(queries, nq, k);
        DeviceGuard g(device_);
        const uint32_t r = static_cast<uint32_t>(4 * k);
        if (n_ == 0) {
            merge_candidates(device_, nullptr, static_cast<uint32_t>(nq), 0, r, 0, 0, 0, nullptr, nullptr, out_cand,
                             stream);
            return;
        }
        finalize(stream);
        const uint32_t nprobe = std::min(nprobe_, nlist_);
        const uint32_t lut_stride = group_lut_stride(m_, ksub_);
        const uint32_t G = group_size(nq * nprobe, r, lut_stride);
        const uint32_t capq = group_capacity(G, r);
        StreamScratch s(plan_bytes(nq, r, false), stream);
        uint8_t* w = s.get();
        // 1-2. probe and plan
        const Plan pl = probe_and_plan(queries, nq, r, G, false, w, stream, probes_in, shared_bound);
        // 3. per (list, query group) approximate scan, R best per (query, list)
        IvfGroupParams p = group_params(queries, pl, r, capq, lut_stride);
        p.codebook = static_cast<const float*>(codebook_.get());
        p.list_codes = static_cast<const uint8_t*>(list_codes_.get());
        p.m = m_;
        p.pq_bits = pq_bits_;
        const size_t smem = group_layout(G, dim_, lut_stride, capq).total;
        const uint64_t max_items = std::min<uint64_t>(pl.npairs, pl.npairs / G + nlist_);
        switch (G) {
            case 8: launch_mb<8>(p, smem, max_items, stream); break;
            case 4: launch_mb<4>(p, smem, max_items, stream); break;
            case 2: launch_mb<2>(p, smem, max_items, stream); break;
            default: launch_mb<1>(p, smem, max_items, stream); break;
        }
        // 4. R best approximate candidates per query across its probed lists
        //    (keys are final approximate distances: no transform, metric 0)
        merge_candidates(device_, pl.part, static_cast<uint32_t>(nq), pl.nprobe, r,
                         static_cast<uint64_t>(pl.nprobe) * r, r, 0, nullptr, nullptr, out_cand, stream);
    }

    // Step 5 (exact_rank, GpuIVFPQIndex.cpp:37-71): exact distances of the
    // R candidates per query on this index's raw rows (slot 0xFFFFFFFF =
    // none), top-k by (distance, slot). cand: [nq][4k] DEVICE.
    void rerank(const float* queries, size_t nq, size_t k, const uint2* cand, float* out_dist, int64_t* out_rows,
                cudaStream_t stream) {
        if (nq == 0 || k == 0) return;
        check_search(queries, nq, k);
        if (cand == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "candidates are null");
        DeviceGuard g(device_);
        const uint32_t r = static_cast<uint32_t>(4 * k);
        uint32_t rp = 1;
        while (rp < r) rp <<= 1;
        constexpr uint32_t warps = 4;
        const size_t rsmem = static_cast<size_t>(warps) * rp * 8;
        allow_dynamic_smem(reinterpret_cast<const void*>(ivfpq_rerank_kernel), rsmem);
        Profiler::Scope prof("ivfpq_rerank", stream, nq * r);
        ivfpq_rerank_kernel<<<static_cast<uint32_t>((nq + warps - 1) / warps), warps * 32, rsmem, stream>>>(
            queries, static_cast<const float*>(vectors_.get()), cand, static_cast<uint32_t>(nq), dim_, r,
            static_cast<uint32_t>(k), rp, static_cast<uint32_t>(n_), metric_, out_dist, out_rows);
        launch_ok("ivf-pq rerank kernel");
    }

private:
    void check_search(const float* queries, size_t nq, size_t k) const {
        if (k > 256) fail(ELIPS_B200_INVALID_ARGUMENT, "k above 256 is not supported (rerank set is 4k)");
        if (nq * nprobe_ > 0x7FFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "too many queries in one call");
        if (queries == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "queries is null");
    }

    void move_row(size_t from, size_t to, cudaStream_t stream) override {
        uint8_t* c = static_cast<uint8_t*>(codes_.get());
        check_cuda(cudaMemcpyAsync(c + to * m_, c + from * m_, m_, cudaMemcpyDeviceToDevice, stream),
                   ELIPS_B200_TRANSFER_FAILED, "code move");
    }

    void grow(size_t rows) override {
        DeviceBuffer c(device_, rows * m_);
        if (n_ > 0)
            check_cuda(cudaMemcpy(c.get(), codes_.get(), n_ * m_, cudaMemcpyDeviceToDevice), ELIPS_B200_TRANSFER_FAILED,
                       "grow copy");
        codes_ = std::move(c);
    }

    void gather_lists(cudaStream_t stream) override {
        list_codes_ = DeviceBuffer(device_, std::max<size_t>(n_, 1) * m_);
        const uint64_t total = static_cast<uint64_t>(n_) * m_;
        Profiler::Scope prof("gather_codes", stream, n_);
        gather_codes_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(
            static_cast<const uint8_t*>(codes_.get()), static_cast<const uint32_t*>(list_rows_.get()), n_, m_,
            static_cast<uint8_t*>(list_codes_.get()));
        launch_ok("gather codes kernel");
    }

    template <int G>
    void launch_mb(const IvfGroupParams& p, size_t smem, uint64_t max_items, cudaStream_t stream) {
        if (pq_bits_ == 8) {
            switch (m_) {
                case 8: return launch_group<G, 8, 8, false>(p, smem, max_items, stream);
                case 16: return launch_group<G, 16, 8, false>(p, smem, max_items, stream);
                case 32: return launch_group<G, 32, 8, false>(p, smem, max_items, stream);
                default: break;
            }
        }
        switch (m_) {
            case 4: return launch_group<G, 4, 0, false>(p, smem, max_items, stream);
            case 8: return launch_group<G, 8, 0, false>(p, smem, max_items, stream);
            case 16: return launch_group<G, 16, 0, false>(p, smem, max_items, stream);
            case 32: return launch_group<G, 32, 0, false>(p, smem, max_items, stream);
            default: return launch_group<G, 0, 0, false>(p, smem, max_items, stream);
        }
    }

    uint32_t m_, ksub_ = 256, pq_bits_ = 8;
    DeviceBuffer codebook_, codes_, list_codes_;
};

// GpuIVFFlatIndex: the probed lists' rows ranked exactly.
class IvfFlatIndex : public IvfLists {
public:
    using IvfLists::IvfLists;

    void add_device(const float* vectors, const uint32_t* assign, size_t n, cudaStream_t stream) {
        if (n == 0) return;
        DeviceGuard g(device_);
        const std::vector<uint32_t> host_assign = append_rows(vectors, assign, n, stream);
        commit_rows(host_assign, stream);
    }

    // search and search_batch (GpuIVFFlatIndex.cpp:84-103, 123-164): results
    // ascending by (distance, gather position); slots, -1 past the candidates.
    void search_device(const float* queries, size_t nq, size_t k, float* out_dist, int64_t* out_rows,
                       cudaStream_t stream) {
        if (nq == 0 || k == 0) return;
        if (k > 1024) fail(ELIPS_B200_INVALID_ARGUMENT, "k above 1024 is not supported");
        if (nq * nprobe_ > 0x7FFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "too many queries in one call");
        if (queries == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "queries is null");
        DeviceGuard g(device_);
        if (n_ == 0) {
            merge_candidates(device_, nullptr, static_cast<uint32_t>(nq), 0, static_cast<uint32_t>(k), 0, 0, 0, out_dist,
                             out_rows, nullptr, stream);
            return;
        }
        finalize(stream);
        const uint32_t r = static_cast<uint32_t>(k);
        const uint32_t nprobe = std::min(nprobe_, nlist_);
        const uint32_t G = group_size(nq * nprobe, r, 0);
        const uint32_t capq = group_capacity(G, r);
        StreamScratch s(plan_bytes(nq, r, true), stream);
        uint8_t* w = s.get();
        const Plan pl = probe_and_plan(queries, nq, r, G, true, w, stream);
        IvfGroupParams p = group_params(queries, pl, r, capq, 0);
        p.list_vecs = static_cast<const float*>(list_vecs_.get());
        const size_t smem = group_layout(G, dim_, 0, capq).total;
        const uint64_t max_items = std::min<uint64_t>(pl.npairs, pl.npairs / G + nlist_);
        switch (G) {
            case 8: launch_group<8, 0, 0, true>(p, smem, max_items, stream); break;
            case 4: launch_group<4, 0, 0, true>(p, smem, max_items, stream); break;
            case 2: launch_group<2, 0, 0, true>(p, smem, max_items, stream); break;
            default: launch_group<1, 0, 0, true>(p, smem, max_items, stream); break;
        }
        // k best over the probed lists by (distance, gather position), then
        // gather positions -> slots
        merge_candidates(device_, pl.part, static_cast<uint32_t>(nq), pl.nprobe, r,
                         static_cast<uint64_t>(pl.nprobe) * r, r, 0, out_dist, out_rows, nullptr, stream);
        const uint64_t total = static_cast<uint64_t>(nq) * k;
        Profiler::Scope prof("ivfflat_slots", stream, total);
        ivf_gather_to_slot_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(
            out_rows, static_cast<uint32_t>(nq), static_cast<uint32_t>(k), pl.probes, pl.nprobe, pl.pair_off,
            static_cast<const uint32_t*>(list_off_.get()), static_cast<const uint32_t*>(list_rows_.get()));
        launch_ok("gather-to-slot kernel");
    }

private:
    void grow(size_t) override {}
    void move_row(size_t, size_t, cudaStream_t) override {}

    void gather_lists(cudaStream_t stream) override {
        list_vecs_ = DeviceBuffer(device_, std::max<size_t>(n_, 1) * dim_ * 4);
        const uint64_t words = static_cast<uint64_t>(n_) * dim_;
        Profiler::Scope prof("gather_rows", stream, n_);
        gather_rows_kernel<<<static_cast<uint32_t>((words + 255) / 256), 256, 0, stream>>>(
            static_cast<const float*>(vectors_.get()), static_cast<const uint32_t*>(list_rows_.get()), n_, dim_,
            static_cast<float*>(list_vecs_.get()));
        launch_ok("gather rows kernel");
    }

    DeviceBuffer list_vecs_;
};

}  // namespace eb

struct elips_b200_ivfpq {
    eb::IvfPqIndex index;
};

struct elips_b200_ivfflat {
    eb::IvfFlatIndex index;
};

namespace {

using eb::guarded;

using eb::OwnedStream;

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

extern "C" {

int elips_b200_ivfpq_create(int device, int metric, uint32_t dimension, uint32_t n_lists, uint32_t nprobe,
                            uint32_t pq_dim, uint32_t pq_bits, const float* centroids, const float* codebook,
                            elips_b200_ivfpq** out) {
    if (out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *out = nullptr;
    return guarded([&] {
        *out = new elips_b200_ivfpq{
            eb::IvfPqIndex(device, metric, dimension, n_lists, nprobe, pq_dim, pq_bits, centroids, codebook)};
    });
}

int elips_b200_ivfpq_add(elips_b200_ivfpq* index, const float* vectors, const uint32_t* assignments,
                         const uint8_t* codes, size_t n) {
    if (index == nullptr || (n > 0 && (vectors == nullptr || assignments == nullptr))) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (n == 0) return;
        eb::IvfPqIndex& ix = index->index;
        eb::DeviceGuard g(ix.device());
        OwnedStream st;
        const size_t vb = up256(n * ix.dim() * 4);
        const size_t ab = up256(n * 4);
        const size_t cb = codes ? n * ix.pq_dim() : 0;
        eb::StreamScratch s(vb + ab + cb + 256, st.s);
        float* dv = reinterpret_cast<float*>(s.get());
        uint32_t* da = reinterpret_cast<uint32_t*>(s.get() + vb);
        uint8_t* dc = codes ? s.get() + vb + ab : nullptr;
        eb::check_cuda(cudaMemcpyAsync(dv, vectors, n * ix.dim() * 4, cudaMemcpyHostToDevice, st.s),
                       ELIPS_B200_TRANSFER_FAILED, "vector upload");
        eb::check_cuda(cudaMemcpyAsync(da, assignments, n * 4, cudaMemcpyHostToDevice, st.s), ELIPS_B200_TRANSFER_FAILED,
                       "assignment upload");
        if (codes != nullptr)
            eb::check_cuda(cudaMemcpyAsync(dc, codes, cb, cudaMemcpyHostToDevice, st.s), ELIPS_B200_TRANSFER_FAILED,
                           "code upload");
        ix.add_device(dv, da, dc, n, st.s);
    });
}

int elips_b200_ivfpq_add_device(elips_b200_ivfpq* index, const float* vectors, const uint32_t* assignments,
                                const uint8_t* codes, size_t n, void* stream) {
    if (index == nullptr || (n > 0 && (vectors == nullptr || assignments == nullptr))) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.add_device(vectors, assignments, codes, n, static_cast<cudaStream_t>(stream)); });
}

int elips_b200_ivfpq_size(const elips_b200_ivfpq* index, size_t* n_out) {
    if (index == nullptr || n_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *n_out = index->index.size();
    return ELIPS_B200_OK;
}

int elips_b200_ivfpq_set_nprobe(elips_b200_ivfpq* index, uint32_t nprobe) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    index->index.set_nprobe(nprobe);
    return ELIPS_B200_OK;
}

int elips_b200_ivfpq_search(elips_b200_ivfpq* index, const float* queries, size_t nq, size_t k, float* out_dist,
                            int64_t* out_rows) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (nq == 0 || k == 0) return;
        eb::IvfPqIndex& ix = index->index;
        eb::DeviceGuard g(ix.device());
        OwnedStream st;
        {
            const size_t qb = up256(nq * ix.dim() * 4);
            const size_t db = up256(nq * k * 4);
            eb::StreamScratch s(qb + db + nq * k * 8 + 256, st.s);
            float* dq = reinterpret_cast<float*>(s.get());
            float* dd = reinterpret_cast<float*>(s.get() + qb);
            int64_t* dr = reinterpret_cast<int64_t*>(s.get() + qb + db);
            eb::check_cuda(cudaMemcpyAsync(dq, queries, nq * ix.dim() * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "query upload");
            ix.search_device(dq, nq, k, dd, dr, st.s);
            eb::check_cuda(cudaMemcpyAsync(out_dist, dd, nq * k * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "distance download");
            eb::check_cuda(cudaMemcpyAsync(out_rows, dr, nq * k * 8, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "ivf-pq search");
    });
}

int elips_b200_ivfpq_search_device(elips_b200_ivfpq* index, const float* queries, size_t nq, size_t k,
                                   float* out_dist, int64_t* out_rows, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.search_device(queries, nq, k, out_dist, out_rows, static_cast<cudaStream_t>(stream)); });
}

int elips_b200_ivfpq_set_list_range(elips_b200_ivfpq* index, uint32_t list_lo, uint32_t list_hi) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.set_list_range(list_lo, list_hi); });
}

int elips_b200_ivfpq_set_owned_lists(elips_b200_ivfpq* index, const uint32_t* mask_words, size_t n_words) {
    if (index == nullptr || mask_words == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.set_owned_lists(mask_words, n_words); });
}

int elips_b200_ivfpq_search_candidates_device(elips_b200_ivfpq* index, const float* queries, size_t nq, size_t k,
                                              uint32_t* out_cand, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_cand == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        index->index.candidates(queries, nq, k, reinterpret_cast<uint2*>(out_cand), static_cast<cudaStream_t>(stream));
    });
}

int elips_b200_ivfpq_probe_device(const elips_b200_ivfpq* index, const float* queries, size_t nq,
                                  uint32_t* probes_out, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && (queries == nullptr || probes_out == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.probe(queries, nq, probes_out, static_cast<cudaStream_t>(stream)); });
}

int elips_b200_ivfpq_search_candidates_probed_device(elips_b200_ivfpq* index, const float* queries, size_t nq,
                                                     size_t k, const uint32_t* probes, uint32_t* out_cand,
                                                     void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || probes == nullptr || out_cand == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        index->index.candidates(queries, nq, k, reinterpret_cast<uint2*>(out_cand), static_cast<cudaStream_t>(stream),
                                probes);
    });
}

int elips_b200_ivfpq_search_candidates_shared_device(elips_b200_ivfpq* index, const float* queries, size_t nq,
                                                     size_t k, const uint32_t* probes, uint32_t* out_cand,
                                                     uint32_t* shared_bound, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_cand == nullptr || shared_bound == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        index->index.candidates(queries, nq, k, reinterpret_cast<uint2*>(out_cand), static_cast<cudaStream_t>(stream),
                                probes, shared_bound);
    });
}

int elips_b200_ivfpq_rerank_device(elips_b200_ivfpq* index, const float* queries, size_t nq, size_t k,
                                   const uint32_t* cand, float* out_dist, int64_t* out_rows, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || cand == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        index->index.rerank(queries, nq, k, reinterpret_cast<const uint2*>(cand), out_dist, out_rows,
                            static_cast<cudaStream_t>(stream));
    });
}

int elips_b200_ivfpq_export(const elips_b200_ivfpq* index, float* centroids_out, uint32_t* assignments_out,
                            float* vectors_out, float* codebook_out, uint8_t* codes_out) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        index->index.export_ivf(centroids_out, assignments_out, vectors_out);
        index->index.export_pq(codebook_out, codes_out);
    });
}

int elips_b200_ivfpq_remove(elips_b200_ivfpq* index, size_t slot) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        OwnedStream st;
        index->index.remove(slot, st.s);
    });
}

int elips_b200_ivfpq_rebuild_codes(elips_b200_ivfpq* index) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        OwnedStream st;
        index->index.rebuild_codes(st.s);
    });
}

int elips_b200_ivfpq_codes_device(const elips_b200_ivfpq* index, uint8_t* codes_out, void* stream) {
    if (index == nullptr || codes_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.read_codes(codes_out, static_cast<cudaStream_t>(stream)); });
}

int elips_b200_ivfpq_destroy(elips_b200_ivfpq* index) {
    if (index == nullptr) return ELIPS_B200_OK;
    return guarded([&] {
        eb::DeviceGuard g(index->index.device());
        delete index;
    });
}

int elips_b200_ivfflat_create(int device, int metric, uint32_t dimension, uint32_t n_lists, uint32_t nprobe,
                              const float* centroids, elips_b200_ivfflat** out) {
    if (out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *out = nullptr;
    return guarded([&] {
        *out = new elips_b200_ivfflat{eb::IvfFlatIndex(device, metric, dimension, n_lists, nprobe, centroids)};
    });
}

int elips_b200_ivfflat_add(elips_b200_ivfflat* index, const float* vectors, const uint32_t* assignments, size_t n) {
    if (index == nullptr || (n > 0 && (vectors == nullptr || assignments == nullptr))) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (n == 0) return;
        eb::IvfFlatIndex& ix = index->index;
        eb::DeviceGuard g(ix.device());
        OwnedStream st;
        const size_t vb = up256(n * ix.dim() * 4);
        eb::StreamScratch s(vb + up256(n * 4), st.s);
        float* dv = reinterpret_cast<float*>(s.get());
        uint32_t* da = reinterpret_cast<uint32_t*>(s.get() + vb);
        eb::check_cuda(cudaMemcpyAsync(dv, vectors, n * ix.dim() * 4, cudaMemcpyHostToDevice, st.s),
                       ELIPS_B200_TRANSFER_FAILED, "vector upload");
        eb::check_cuda(cudaMemcpyAsync(da, assignments, n * 4, cudaMemcpyHostToDevice, st.s), ELIPS_B200_TRANSFER_FAILED,
                       "assignment upload");
        ix.add_device(dv, da, n, st.s);
    });
}

int elips_b200_ivfflat_add_device(elips_b200_ivfflat* index, const float* vectors, const uint32_t* assignments,
                                  size_t n, void* stream) {
    if (index == nullptr || (n > 0 && (vectors == nullptr || assignments == nullptr))) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.add_device(vectors, assignments, n, static_cast<cudaStream_t>(stream)); });
}

int elips_b200_ivfflat_export(const elips_b200_ivfflat* index, float* centroids_out, uint32_t* assignments_out,
                              float* vectors_out) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.export_ivf(centroids_out, assignments_out, vectors_out); });
}

int elips_b200_ivfflat_remove(elips_b200_ivfflat* index, size_t slot) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        OwnedStream st;
        index->index.remove(slot, st.s);
    });
}

int elips_b200_ivfflat_size(const elips_b200_ivfflat* index, size_t* n_out) {
    if (index == nullptr || n_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *n_out = index->index.size();
    return ELIPS_B200_OK;
}

int elips_b200_ivfflat_set_nprobe(elips_b200_ivfflat* index, uint32_t nprobe) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    index->index.set_nprobe(nprobe);
    return ELIPS_B200_OK;
}

int elips_b200_ivfflat_search(elips_b200_ivfflat* index, const float* queries, size_t nq, size_t k,
                              float* out_dist, int64_t* out_rows) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (nq == 0 || k == 0) return;
        eb::IvfFlatIndex& ix = index->index;
        eb::DeviceGuard g(ix.device());
        OwnedStream st;
        {
            const size_t qb = up256(nq * ix.dim() * 4);
            const size_t db = up256(nq * k * 4);
            eb::StreamScratch s(qb + db + nq * k * 8 + 256, st.s);
            float* dq = reinterpret_cast<float*>(s.get());
            float* dd = reinterpret_cast<float*>(s.get() + qb);
            int64_t* dr = reinterpret_cast<int64_t*>(s.get() + qb + db);
            eb::check_cuda(cudaMemcpyAsync(dq, queries, nq * ix.dim() * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "query upload");
            ix.search_device(dq, nq, k, dd, dr, st.s);
            eb::check_cuda(cudaMemcpyAsync(out_dist, dd, nq * k * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "distance download");
            eb::check_cuda(cudaMemcpyAsync(out_rows, dr, nq * k * 8, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "ivf-flat search");
    });
}

int elips_b200_ivfflat_search_device(elips_b200_ivfflat* index, const float* queries, size_t nq, size_t k,
                                     float* out_dist, int64_t* out_rows, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.search_device(queries, nq, k, out_dist, out_rows, static_cast<cudaStream_t>(stream)); });
}

int elips_b200_ivfflat_destroy(elips_b200_ivfflat* index) {
    if (index == nullptr) return ELIPS_B200_OK;
    return guarded([&] {
        eb::DeviceGuard g(index->index.device());
        delete index;
    });
}

}  // extern "C"
