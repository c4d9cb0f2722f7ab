// Host side of the bit-exact SIMT paths: GpuPort's distance / top-k
// primitives and the ExactIndex-with-Quantizer scans (PQ, OPQ, sq8).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include <cub/device/device_segmented_radix_sort.cuh>

#include "../../include/elips_b200.h"
#include "engine.cuh"
#include "capi_util.cuh"
#include "train.cuh"
#include "profiler.cuh"
#include "scan_kernels.cuh"

namespace eb {
namespace {

constexpr uint32_t kMaxK = 1024;

uint32_t pow2_at_least(uint32_t x) {
    uint32_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

uint32_t btk_cap(uint32_t k) { return (k + kScanThreads + 31u) / 32u * 32u; }

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

void launch_check(const char* what) { check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, what); }

// Number of row splits for a scan over n rows with `cta_rows` CTAs per split
// column: aim for ~4 CTAs per SM, keep >= 1024 rows per split.
uint32_t scan_splits(uint32_t n, uint32_t ctas_per_split, int num_sms) {
    const uint32_t want = std::max<uint32_t>(1, (4u * num_sms + ctas_per_split - 1) / ctas_per_split);
    const uint32_t max_by_rows = std::max<uint32_t>(1, n / 1024u);
    return std::min<uint32_t>({want, max_by_rows, 4096u});
}

}  // namespace

void compute_distances_device(int device, const float* q, const float* db, float* out, size_t nq, size_t nb,
                              size_t d, int metric, cudaStream_t stream) {
    if (nq == 0 || nb == 0) return;
    if (metric < 0 || metric > 2) fail(ELIPS_B200_UNSUPPORTED_METRIC, "unknown metric");
    if (d == 0) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension is zero");
    if (nb > 0xFFFFFFFFull || nq > 65535ull * kDistQ) fail(ELIPS_B200_INVALID_ARGUMENT, "batch too large");
    DeviceGuard g(device);
    device_props(device);
    const dim3 grid(static_cast<uint32_t>((nb + kDistRows - 1) / kDistRows), static_cast<uint32_t>((nq + kDistQ - 1) / kDistQ));
    Profiler::Scope prof("distances", stream, static_cast<uint64_t>(nq) * nb);
    distances_kernel<<<grid, kDistRows, 0, stream>>>(q, db, static_cast<uint32_t>(nq), static_cast<uint32_t>(nb),
                                                    static_cast<uint32_t>(d), metric, out);
    launch_check("distances kernel");
}

namespace {

__global__ void column_index_kernel(uint32_t* __restrict__ idx, uint64_t total, uint32_t nb) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t < total) idx[t] = static_cast<uint32_t>(t % nb);
}

__global__ void row_offsets_kernel(uint64_t* __restrict__ off, uint32_t rows, uint64_t nb) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t <= rows) off[t] = static_cast<uint64_t>(t) * nb;
}

__global__ void take_first_k_kernel(const float* __restrict__ sval, const uint32_t* __restrict__ sidx, uint32_t rows,
                                    uint64_t nb, uint64_t k, float* __restrict__ val, uint32_t* __restrict__ idx) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<uint64_t>(rows) * k) return;
    const uint64_t q = t / k, i = t % k;
    const bool in = i < nb;
    val[t] = in ? sval[q * nb + i] : __int_as_float(0x7f800000);
    idx[t] = in ? sidx[q * nb + i] : 0xFFFFFFFFu;
}

// GpuPort::top_k for k above the block select's reach: every row sorted by
// value with a stable segmented radix sort (columns enter in order, so equal
// values keep ascending column order, the port's tie rule), then the first k.
// Rows go in chunks of at most 2^30 values.
void top_k_sorted(const float* dist, uint32_t* idx, float* val, size_t nq, size_t nb, size_t k, cudaStream_t stream) {
    const size_t rows_per = std::max<size_t>(1, (size_t{1} << 30) / std::max<size_t>(nb, 1));
    for (size_t q0 = 0; q0 < nq; q0 += rows_per) {
        const uint32_t rows = static_cast<uint32_t>(std::min(rows_per, nq - q0));
        const uint64_t total = static_cast<uint64_t>(rows) * nb;
        size_t temp = 0;
        cub::DeviceSegmentedRadixSort::SortPairs(nullptr, temp, static_cast<const float*>(nullptr),
                                                 static_cast<float*>(nullptr), static_cast<const uint32_t*>(nullptr),
                                                 static_cast<uint32_t*>(nullptr), static_cast<int64_t>(total),
                                                 static_cast<int64_t>(rows), static_cast<const uint64_t*>(nullptr),
                                                 static_cast<const uint64_t*>(nullptr), 0, 32, stream);
        const size_t a_val = align256(total * 4), a_idx = align256(total * 4), a_off = align256((rows + 1ull) * 8);
        StreamScratch s(a_val + 2 * a_idx + a_off + align256(temp), stream);
        float* sval = reinterpret_cast<float*>(s.get());
        uint32_t* in_idx = reinterpret_cast<uint32_t*>(s.get() + a_val);
        uint32_t* sidx = reinterpret_cast<uint32_t*>(s.get() + a_val + a_idx);
        uint64_t* off = reinterpret_cast<uint64_t*>(s.get() + a_val + 2 * a_idx);
        void* tmp = s.get() + a_val + 2 * a_idx + a_off;
        Profiler::Scope prof("topk_sorted", stream, total);
        column_index_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(
            in_idx, total, static_cast<uint32_t>(nb));
        row_offsets_kernel<<<(rows + 256) / 256, 256, 0, stream>>>(off, rows, nb);
        launch_check("top-k sort setup");
        check_cuda(cub::DeviceSegmentedRadixSort::SortPairs(tmp, temp, dist + q0 * nb, sval, in_idx, sidx,
                                                            static_cast<int64_t>(total), static_cast<int64_t>(rows),
                                                            off, off + 1, 0, 32, stream),
                   ELIPS_B200_KERNEL_LAUNCH_FAILED, "segmented sort");
        const uint64_t outs = static_cast<uint64_t>(rows) * k;
        take_first_k_kernel<<<static_cast<uint32_t>((outs + 255) / 256), 256, 0, stream>>>(
            sval, sidx, rows, nb, k, val + q0 * k, idx + q0 * k);
        launch_check("top-k take");
    }
}

}  // namespace

void top_k_device(int device, const float* dist, uint32_t* idx, float* val, size_t nq, size_t nb, size_t k,
                  cudaStream_t stream) {
    if (nq == 0 || k == 0) return;
    if (nb > 0xFFFFFFFEull || nq > 0x7FFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "batch too large");
    DeviceGuard g(device);
    device_props(device);
    if (k > kMaxK) {
        if (nb == 0) fail(ELIPS_B200_INVALID_ARGUMENT, "empty distance rows");
        top_k_sorted(dist, idx, val, nq, nb, k, stream);
        return;
    }
    if (k <= 256) {  // one warp per row
        top_k_rows_warp(device, dist, idx, val, nq, nb, k, stream);
        return;
    }
    const uint32_t cap = btk_cap(static_cast<uint32_t>(k));
    const uint32_t kp = pow2_at_least(static_cast<uint32_t>(k));
    const size_t smem = btk_bytes(cap) + static_cast<size_t>(kp) * 8;
    allow_dynamic_smem(reinterpret_cast<const void*>(topk_rows_kernel), smem);
    Profiler::Scope prof("topk_rows", stream, static_cast<uint64_t>(nq) * nb);
    topk_rows_kernel<<<static_cast<uint32_t>(nq), kScanThreads, smem, stream>>>(
        dist, static_cast<uint32_t>(nq), static_cast<uint32_t>(nb), static_cast<uint32_t>(k), cap, kp, idx, val);
    launch_check("top-k kernel");
}

void normalize_rows_device(int device, const float* in, float* out, size_t n, size_t d, cudaStream_t stream) {
    if (n == 0 || d == 0) return;
    if (d > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must be in [1, 65535]");
    DeviceGuard g(device);
    device_props(device);
    const uint64_t blocks = (n + kNormRows - 1) / kNormRows;
    if (blocks > 0x7FFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "too many rows in one call");
    Profiler::Scope prof("normalize_rows", stream, n);
    normalize_rows_kernel<<<static_cast<uint32_t>(blocks), 256, 0, stream>>>(in, out, n, static_cast<uint32_t>(d));
    launch_check("normalize kernel");
}

// ExactIndex with a Quantizer attached, codes resident on the device.
class QuantIndex {
public:
    QuantIndex(int device, int codec, int metric, uint32_t dim, uint32_t pq_dim, uint32_t pq_bits,
               const float* params, const float* rotation)
        : device_(device), codec_(codec), metric_(metric), dim_(dim), pq_dim_(pq_dim), pq_bits_(pq_bits) {
        if (metric < 0 || metric > 2) fail(ELIPS_B200_UNSUPPORTED_METRIC, "unknown metric");
        if (dim == 0 || dim > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must be in [1, 65535]");
        if (params == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "codec parameters are null");
        device_props(device);
        DeviceGuard g(device);
        if (codec == ELIPS_B200_CODEC_SQ8) {
            code_bytes_ = dim;
            params_ = DeviceBuffer(device, 2ull * dim * sizeof(float));
            check_cuda(cudaMemcpy(params_.get(), params, 2ull * dim * sizeof(float), cudaMemcpyHostToDevice),
                       ELIPS_B200_TRANSFER_FAILED, "sq8 parameters");
        } else if (codec == ELIPS_B200_CODEC_PQ || codec == ELIPS_B200_CODEC_OPQ) {
            if (pq_dim == 0 || dim % pq_dim != 0 || pq_bits < 4 || pq_bits > 8)
                fail(ELIPS_B200_INVALID_ARGUMENT, "pq_dim must divide the dimension and pq_bits be in [4, 8]");
            if ((codec == ELIPS_B200_CODEC_OPQ) != (rotation != nullptr))
                fail(ELIPS_B200_INVALID_ARGUMENT, "OPQ needs a rotation and PQ must not have one");
            code_bytes_ = pq_dim;
            ksub_ = 1u << pq_bits;
            const size_t cb = static_cast<size_t>(pq_dim) * ksub_ * (dim / pq_dim);
            params_ = DeviceBuffer(device, cb * sizeof(float));
            check_cuda(cudaMemcpy(params_.get(), params, cb * sizeof(float), cudaMemcpyHostToDevice),
                       ELIPS_B200_TRANSFER_FAILED, "pq codebook");
            if (rotation != nullptr) {
                rotation_ = DeviceBuffer(device, static_cast<size_t>(dim) * dim * sizeof(float));
                check_cuda(cudaMemcpy(rotation_.get(), rotation, static_cast<size_t>(dim) * dim * sizeof(float),
                                      cudaMemcpyHostToDevice),
                           ELIPS_B200_TRANSFER_FAILED, "opq rotation");
            }
        } else {
            fail(ELIPS_B200_INVALID_ARGUMENT, "unknown codec");
        }
    }

    int device() const { return device_; }
    size_t size() const { return n_; }
    uint32_t dim() const { return dim_; }

    void add_codes_device(const uint8_t* codes, size_t n, cudaStream_t stream) {
        reserve(n_ + n);
        check_cuda(cudaMemcpyAsync(static_cast<uint8_t*>(codes_.get()) + n_ * code_bytes_, codes, n * code_bytes_,
                                   cudaMemcpyDeviceToDevice, stream),
                   ELIPS_B200_TRANSFER_FAILED, "code copy");
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_TRANSFER_FAILED, "code copy");
        n_ += n;
    }

    void add_codes_host(const uint8_t* codes, size_t n) {
        if (n == 0) return;
        DeviceGuard g(device_);
        reserve(n_ + n);
        check_cuda(cudaMemcpy(static_cast<uint8_t*>(codes_.get()) + n_ * code_bytes_, codes, n * code_bytes_,
                              cudaMemcpyHostToDevice),
                   ELIPS_B200_TRANSFER_FAILED, "code upload");
        n_ += n;
    }

    // Encodes fp32 rows (device) with the codec's own encode and appends them.
    void encode_add_device(const float* rows, size_t n, cudaStream_t stream) {
        if (n == 0) return;
        DeviceGuard g(device_);
        reserve(n_ + n);
        uint8_t* dst = static_cast<uint8_t*>(codes_.get()) + n_ * code_bytes_;
        const float* src = rows;
        StreamScratch rot(rotation_.get() ? n * dim_ * sizeof(float) : 0, stream);
        if (rotation_.get() != nullptr) {
            const uint64_t total = static_cast<uint64_t>(n) * dim_;
            Profiler::Scope prof("rotate_rows", stream, n);
            rotate_rows_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(
                static_cast<const float*>(rotation_.get()), rows, n, dim_, reinterpret_cast<float*>(rot.get()));
            launch_check("rotate kernel");
            src = reinterpret_cast<const float*>(rot.get());
        }
        if (codec_ == ELIPS_B200_CODEC_SQ8) {
            const uint64_t total = static_cast<uint64_t>(n) * dim_;
            const float* mins = static_cast<const float*>(params_.get());
            Profiler::Scope prof("sq8_encode", stream, n);
            sq8_encode_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(src, mins, mins + dim_, n,
                                                                                           dim_, dst);
        } else {
            pq_encode_device(src, n, dim_, pq_dim_, ksub_, static_cast<const float*>(params_.get()), dst, stream);
        }
        launch_check("encode kernel");
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "encode");
        n_ += n;
    }

    void search_device(const float* queries, size_t nq, size_t k, float* out_dist, int64_t* out_rows,
                       cudaStream_t stream) const {
        if (nq == 0 || k == 0) return;
        if (k > kMaxK) fail(ELIPS_B200_INVALID_ARGUMENT, "k above 1024 is not supported");
        if (nq > 65535ull * kPqQueriesPerCta) fail(ELIPS_B200_INVALID_ARGUMENT, "too many queries in one call");
        DeviceGuard g(device_);
        const DeviceProps& props = device_props(device_);
        if (n_ == 0) {
            merge_candidates(device_, nullptr, static_cast<uint32_t>(nq), 0, static_cast<uint32_t>(k), 0, 0, 0, out_dist,
                             out_rows, nullptr, stream);
            return;
        }
        const uint32_t n = static_cast<uint32_t>(n_);
        const uint32_t cap = btk_cap(static_cast<uint32_t>(k));
        const bool sq8 = codec_ == ELIPS_B200_CODEC_SQ8;
        const size_t lut_floats = sq8 ? static_cast<size_t>(dim_) * 256 : static_cast<size_t>(pq_dim_) * ksub_;
        const uint32_t ctas_per_split = sq8 ? static_cast<uint32_t>(nq)
                                            : static_cast<uint32_t>((nq + kPqQueriesPerCta - 1) / kPqQueriesPerCta);
        const uint32_t splits = scan_splits(n, ctas_per_split, props.num_sms);
        const size_t rot_bytes = rotation_.get() ? align256(nq * dim_ * sizeof(float)) : 0;
        const size_t lut_bytes = align256(nq * lut_floats * sizeof(float));
        const size_t part_bytes = align256(nq * splits * k * sizeof(uint2));
        StreamScratch scratch(rot_bytes + lut_bytes + part_bytes, stream);
        const float* q = queries;
        if (rot_bytes) {
            float* rq = reinterpret_cast<float*>(scratch.get());
            const uint64_t total = static_cast<uint64_t>(nq) * dim_;
            Profiler::Scope prof("rotate_rows", stream, nq);
            rotate_rows_kernel<<<static_cast<uint32_t>((total + 255) / 256), 256, 0, stream>>>(
                static_cast<const float*>(rotation_.get()), queries, nq, dim_, rq);
            launch_check("rotate kernel");
            q = rq;
        }
        float* lut = reinterpret_cast<float*>(scratch.get() + rot_bytes);
        uint2* part = reinterpret_cast<uint2*>(scratch.get() + rot_bytes + lut_bytes);
        const uint64_t lut_total = nq * lut_floats;
        const uint32_t lut_blocks = static_cast<uint32_t>((lut_total + 255) / 256);
        if (sq8) {
            const float* mins = static_cast<const float*>(params_.get());
            {
                Profiler::Scope prof("sq8_lut", stream, nq);
                sq8_lut_kernel<<<lut_blocks, 256, 0, stream>>>(q, mins, mins + dim_, static_cast<uint32_t>(nq), dim_,
                                                              metric_, lut);
                launch_check("sq8 lut kernel");
            }
            const bool in_smem = dim_ <= 192;
            const size_t smem = btk_bytes(cap) + (in_smem ? static_cast<size_t>(dim_) * 256 * sizeof(float) : 0);
            allow_dynamic_smem(reinterpret_cast<const void*>(sq8_scan_kernel), smem);
            Profiler::Scope prof("sq8_scan", stream, static_cast<uint64_t>(nq) * n);
            sq8_scan_kernel<<<dim3(splits, static_cast<uint32_t>(nq)), kScanThreads, smem, stream>>>(
                lut, static_cast<const uint8_t*>(codes_.get()), n, dim_, metric_, static_cast<uint32_t>(k), cap, splits,
                in_smem ? 1 : 0, part);
            launch_check("sq8 scan kernel");
        } else {
            {
                Profiler::Scope prof("pq_lut", stream, nq);
                pq_lut_kernel<<<lut_blocks, 256, 0, stream>>>(q, static_cast<const float*>(params_.get()),
                                                             static_cast<uint32_t>(nq), dim_, pq_dim_, ksub_, metric_, lut);
                launch_check("pq lut kernel");
            }
            const size_t smem = kPqQueriesPerCta * (lut_floats * sizeof(float) + btk_bytes(cap));
            if (smem > device_props(device_).max_smem_optin)
                fail(ELIPS_B200_INVALID_ARGUMENT, "pq_dim x 2^pq_bits too large for the scan kernel");
            allow_dynamic_smem(reinterpret_cast<const void*>(pq_scan_kernel), smem);
            const dim3 grid(splits, static_cast<uint32_t>((nq + kPqQueriesPerCta - 1) / kPqQueriesPerCta));
            Profiler::Scope prof("pq_scan", stream, static_cast<uint64_t>(nq) * n);
            pq_scan_kernel<<<grid, kScanThreads, smem, stream>>>(lut, static_cast<const uint8_t*>(codes_.get()), n,
                                                                 static_cast<uint32_t>(nq), pq_dim_, ksub_, metric_,
                                                                 static_cast<uint32_t>(k), cap, splits, part);
            launch_check("pq scan kernel");
        }
        // Keys are final lut_distance values: the merge applies no transform (0).
        merge_candidates(device_, part, static_cast<uint32_t>(nq), splits, static_cast<uint32_t>(k),
                         static_cast<uint64_t>(splits) * k, k, 0, out_dist, out_rows, nullptr, stream);
    }

private:
    void reserve(size_t rows) {
        if (rows <= capacity_) return;
        if (rows >= 0xFFFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "index limited to 2^32-2 rows");
        const size_t cap = std::max<size_t>(rows, capacity_ + capacity_ / 2);
        DeviceBuffer nb(device_, cap * code_bytes_);
        if (n_ > 0)
            check_cuda(cudaMemcpy(nb.get(), codes_.get(), n_ * code_bytes_, cudaMemcpyDeviceToDevice),
                       ELIPS_B200_TRANSFER_FAILED, "grow copy");
        codes_ = std::move(nb);
        capacity_ = cap;
    }

    int device_, codec_, metric_;
    uint32_t dim_, pq_dim_, pq_bits_, ksub_ = 256, code_bytes_ = 0;
    size_t n_ = 0, capacity_ = 0;
    DeviceBuffer params_, rotation_, codes_;
};

}  // namespace eb

struct elips_b200_quant {
    eb::QuantIndex index;
};

namespace {

using eb::guarded;

size_t align_up(size_t x) { return (x + 255) / 256 * 256; }

using eb::OwnedStream;

}  // namespace

extern "C" {

int elips_b200_normalize_rows(int device, const float* in, float* out, size_t n, size_t d, int pointers_on_device,
                              void* stream) {
    if (n > 0 && d > 0 && (in == nullptr || out == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::normalize_rows_device(device, in, out, n, d, static_cast<cudaStream_t>(stream));
            return;
        }
        if (n == 0 || d == 0) return;
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            eb::StreamScratch s(2 * n * d * 4 + 512, st.s);
            float* din = reinterpret_cast<float*>(s.get());
            float* dout = din + n * d;
            eb::check_cuda(cudaMemcpyAsync(din, in, n * d * 4, cudaMemcpyHostToDevice, st.s), ELIPS_B200_TRANSFER_FAILED,
                           "row upload");
            eb::normalize_rows_device(device, din, dout, n, d, st.s);
            eb::check_cuda(cudaMemcpyAsync(out, dout, n * d * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "normalize");
    });
}

int elips_b200_compute_distances_batch(int device, const float* queries, const float* database,
                                       float* distances_out, size_t nq, size_t nb, size_t dim, int metric,
                                       int pointers_on_device, void* stream) {
    if (nq > 0 && nb > 0 && (queries == nullptr || database == nullptr || distances_out == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::compute_distances_device(device, queries, database, distances_out, nq, nb, dim, metric,
                                         static_cast<cudaStream_t>(stream));
            return;
        }
        if (nq == 0 || nb == 0) return;
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            eb::StreamScratch s((nq + nb) * dim * 4 + nq * nb * 4 + 512, st.s);
            float* dq = reinterpret_cast<float*>(s.get());
            float* ddb = dq + nq * dim;
            float* dout = ddb + nb * dim;
            eb::check_cuda(cudaMemcpyAsync(dq, queries, nq * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "query upload");
            eb::check_cuda(cudaMemcpyAsync(ddb, database, nb * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "database upload");
            eb::compute_distances_device(device, dq, ddb, dout, nq, nb, dim, metric, st.s);
            eb::check_cuda(cudaMemcpyAsync(distances_out, dout, nq * nb * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "distance download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "distances");
    });
}

namespace {

// Row-major C[m][n] = op(A) op(B) in fp32, 64 x 64 output tile per block of
// 256 threads (4 x 4 per thread), k staged 16 at a time in shared memory.
// op(A)[i][p] = trans_a ? A[p][i] : A[i][p] (A is m x kk, or kk x m);
// op(B)[p][j] = trans_b ? B[j][p] : B[p][j].
__global__ void __launch_bounds__(256) gemm_fp32_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                        float* __restrict__ C, uint32_t m, uint32_t n, uint32_t kk,
                                                        int trans_a, int trans_b) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const uint32_t tx = threadIdx.x & 15u, ty = threadIdx.x >> 4;
    const uint32_t i0 = blockIdx.y * 64u, j0 = blockIdx.x * 64u;
    float acc[4][4] = {};
    for (uint32_t p0 = 0; p0 < kk; p0 += 16) {
        for (uint32_t e = threadIdx.x; e < 16u * 64u; e += 256u) {
            const uint32_t pp = e / 64u, ii = e % 64u;
            const uint32_t i = i0 + ii, j = j0 + ii, p = p0 + pp;
            float av = 0.0f, bv = 0.0f;
            if (i < m && p < kk) av = trans_a ? A[static_cast<size_t>(p) * m + i] : A[static_cast<size_t>(i) * kk + p];
            if (j < n && p < kk) bv = trans_b ? B[static_cast<size_t>(j) * kk + p] : B[static_cast<size_t>(p) * n + j];
            As[pp][ii] = av;
            Bs[pp][ii] = bv;
        }
        __syncthreads();
#pragma unroll
        for (uint32_t pp = 0; pp < 16; ++pp) {
            float a[4], b[4];
#pragma unroll
            for (uint32_t r = 0; r < 4; ++r) a[r] = As[pp][ty * 4u + r];
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) b[c] = Bs[pp][tx * 4u + c];
#pragma unroll
            for (uint32_t r = 0; r < 4; ++r)
#pragma unroll
                for (uint32_t c = 0; c < 4; ++c) acc[r][c] = fmaf(a[r], b[c], acc[r][c]);
        }
        __syncthreads();
    }
#pragma unroll
    for (uint32_t r = 0; r < 4; ++r)
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) {
            const uint32_t i = i0 + ty * 4u + r, j = j0 + tx * 4u + c;
            if (i < m && j < n) C[static_cast<size_t>(i) * n + j] = acc[r][c];
        }
}

void gemm_fp32_device(const float* a, const float* b, float* c, size_t m, size_t n, size_t kk, int trans_a,
                      int trans_b, cudaStream_t stream) {
    if (m == 0 || n == 0) return;
    if (m > 0x7FFFFFFFull || n > 0x7FFFFFFFull || kk > 0x7FFFFFFFull)
        eb::fail(ELIPS_B200_INVALID_ARGUMENT, "GEMM dimensions above 2^31");
    const dim3 grid(static_cast<uint32_t>((n + 63) / 64), static_cast<uint32_t>((m + 63) / 64));
    gemm_fp32_kernel<<<grid, 256, 0, stream>>>(a, b, c, static_cast<uint32_t>(m), static_cast<uint32_t>(n),
                                               static_cast<uint32_t>(kk), trans_a, trans_b);
    eb::check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "gemm launch");
}

}  // namespace

int elips_b200_gemm_fp32(int device, const float* a, const float* b, float* c, size_t m, size_t n, size_t k_inner,
                         int trans_a, int trans_b, int pointers_on_device, void* stream) {
    if (m > 0 && n > 0 && (a == nullptr || b == nullptr || c == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        eb::DeviceGuard g(device);
        if (pointers_on_device) {
            gemm_fp32_device(a, b, c, m, n, k_inner, trans_a, trans_b, static_cast<cudaStream_t>(stream));
            return;
        }
        if (m == 0 || n == 0) return;
        OwnedStream st;
        {
            eb::StreamScratch s((m * k_inner + k_inner * n + m * n) * 4 + 512, st.s);
            float* da = reinterpret_cast<float*>(s.get());
            float* db = da + m * k_inner;
            float* dc = db + k_inner * n;
            eb::check_cuda(cudaMemcpyAsync(da, a, m * k_inner * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "gemm upload");
            eb::check_cuda(cudaMemcpyAsync(db, b, k_inner * n * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "gemm upload");
            gemm_fp32_device(da, db, dc, m, n, k_inner, trans_a, trans_b, st.s);
            eb::check_cuda(cudaMemcpyAsync(c, dc, m * n * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "gemm download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "gemm");
    });
}

int elips_b200_top_k(int device, const float* distances, uint32_t* indices_out, float* values_out, size_t nq,
                     size_t nb, size_t k, int pointers_on_device, void* stream) {
    if (nq > 0 && k > 0 && (indices_out == nullptr || values_out == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && nb > 0 && distances == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::top_k_device(device, distances, indices_out, values_out, nq, nb, k, static_cast<cudaStream_t>(stream));
            return;
        }
        if (nq == 0 || k == 0) return;
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            eb::StreamScratch s(nq * nb * 4 + nq * k * 8 + 512, st.s);
            float* dd = reinterpret_cast<float*>(s.get());
            uint32_t* di = reinterpret_cast<uint32_t*>(dd + nq * nb);
            float* dv = reinterpret_cast<float*>(di + nq * k);
            eb::check_cuda(cudaMemcpyAsync(dd, distances, nq * nb * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "distance upload");
            eb::top_k_device(device, dd, di, dv, nq, nb, k, st.s);
            eb::check_cuda(cudaMemcpyAsync(indices_out, di, nq * k * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "index download");
            eb::check_cuda(cudaMemcpyAsync(values_out, dv, nq * k * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "value download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "top_k");
    });
}

int elips_b200_quant_create(int device, int codec, int metric, uint32_t dimension, uint32_t pq_dim,
                            uint32_t pq_bits, const float* params, const float* rotation,
                            elips_b200_quant** out) {
    if (out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *out = nullptr;
    return guarded([&] {
        *out = new elips_b200_quant{eb::QuantIndex(device, codec, metric, dimension, pq_dim, pq_bits, params, rotation)};
    });
}

int elips_b200_quant_add(elips_b200_quant* index, const float* rows, size_t n) {
    if (index == nullptr || (n > 0 && rows == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (n == 0) return;
        eb::DeviceGuard g(index->index.device());
        OwnedStream st;
        const size_t bytes = n * index->index.dim() * sizeof(float);
        eb::StreamScratch s(bytes, st.s);
        eb::check_cuda(cudaMemcpyAsync(s.get(), rows, bytes, cudaMemcpyHostToDevice, st.s), ELIPS_B200_TRANSFER_FAILED,
                       "row upload");
        index->index.encode_add_device(reinterpret_cast<const float*>(s.get()), n, st.s);
    });
}

int elips_b200_quant_add_codes(elips_b200_quant* index, const uint8_t* codes, size_t n) {
    if (index == nullptr || (n > 0 && codes == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.add_codes_host(codes, n); });
}

int elips_b200_quant_size(const elips_b200_quant* index, size_t* n_out) {
    if (index == nullptr || n_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *n_out = index->index.size();
    return ELIPS_B200_OK;
}

int elips_b200_quant_search(const elips_b200_quant* index, const float* queries, size_t nq, size_t k,
                            float* out_dist, int64_t* out_rows) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (nq == 0 || k == 0) return;
        const eb::QuantIndex& ix = index->index;
        eb::DeviceGuard g(ix.device());
        OwnedStream st;
        {
            const size_t qb = nq * ix.dim() * sizeof(float);
            const size_t ob = nq * k;
            eb::StreamScratch s(align_up(qb) + ob * 12 + 512, st.s);
            float* dq = reinterpret_cast<float*>(s.get());
            float* dd = reinterpret_cast<float*>(s.get() + align_up(qb));
            int64_t* dr = reinterpret_cast<int64_t*>(s.get() + align_up(qb) + align_up(ob * 4));
            eb::check_cuda(cudaMemcpyAsync(dq, queries, qb, cudaMemcpyHostToDevice, st.s), ELIPS_B200_TRANSFER_FAILED,
                           "query upload");
            ix.search_device(dq, nq, k, dd, dr, st.s);
            eb::check_cuda(cudaMemcpyAsync(out_dist, dd, ob * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "distance download");
            eb::check_cuda(cudaMemcpyAsync(out_rows, dr, ob * 8, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "quantized search");
    });
}

int elips_b200_quant_search_device(const elips_b200_quant* index, const float* queries, size_t nq, size_t k,
                                   float* out_dist, int64_t* out_rows, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.search_device(queries, nq, k, out_dist, out_rows, static_cast<cudaStream_t>(stream)); });
}

int elips_b200_quant_destroy(elips_b200_quant* index) {
    if (index == nullptr) return ELIPS_B200_OK;
    return guarded([&] {
        eb::DeviceGuard g(index->index.device());
        delete index;
    });
}

}  // extern "C"
