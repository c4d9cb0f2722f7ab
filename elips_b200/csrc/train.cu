// Device index build: k-means (quant::detail::kmeans), PQ codebook training
// (quant::detail::train_pq_codebook), IVF centroid training and assignment
// (IvfIndexState::train_centroids / assign_vectors_to_centroids), and the whole
// IVF-PQ model build of GpuIVFPQIndex (rebuild_from_current_data followed by
// rebuild_codes). Results are bit-identical to the reference's CPU loops.
//
// One Lloyd round on the device:
//   nearest_centroid_kernel   keys = batch * K + nearest centroid
//   cub::DeviceRadixSort      (key, row) pairs, stable: each centroid's rows
//                             come out in ascending row order
//   segment_bounds_kernel     [start, end) per key
//   centroid_update_kernel    ordered member sums -> new centroids
// A "batch" is one independent k-means over its own columns of the same rows
// (PQ: one per subspace, all trained by the same launches).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include <cub/device/device_radix_sort.cuh>

#include "../../include/elips_b200.h"
#include "engine.cuh"
#include "capi_util.cuh"
#include "ivfpq_kernels.cuh"
#include "profiler.cuh"
#include "scan_kernels.cuh"
#include "train.cuh"
#include "train_kernels.cuh"

namespace eb {
namespace {

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

void launch_ok(const char* what) { check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, what); }

uint32_t blocks_for(uint64_t total, uint32_t threads) {
    const uint64_t b = (total + threads - 1) / threads;
    if (b > 0x7FFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "training problem too large for one launch");
    return static_cast<uint32_t>(std::max<uint64_t>(b, 1));
}

int key_bits(uint64_t max_key) {
    int bits = 1;
    while (bits < 32 && (max_key >> bits) != 0) ++bits;
    return bits;
}

// Rows of the problem: `n` rows of pitch `ld` floats; batch b uses columns
// [b * batch_cols, b * batch_cols + d).
struct TrainRows {
    const float* rows;
    uint64_t ld, n;
    uint32_t d, batch, batch_cols;
};

void launch_nearest(int mode, const TrainRows& p, const float* cents, uint32_t K, uint32_t key_stride, uint32_t* keys,
                    const uint32_t* done, cudaStream_t stream, float* best = nullptr) {
    const uint64_t tiles = (p.n + kAsgRows - 1) / kAsgRows;
    if (tiles > 0x7FFFFFFFull || p.batch > 65535u) fail(ELIPS_B200_INVALID_ARGUMENT, "too many rows in one call");
    const dim3 grid(static_cast<uint32_t>(tiles), p.batch);
    Profiler::Scope prof("nearest_centroid", stream, p.n * p.batch);
    switch (mode) {
        case kTrainSqL2:
            nearest_centroid_kernel<kTrainSqL2><<<grid, 256, 0, stream>>>(p.rows, p.ld, p.n, p.d, p.batch_cols, cents,
                                                                         K, key_stride, keys, done, best);
            break;
        case kTrainL2:
            nearest_centroid_kernel<kTrainL2><<<grid, 256, 0, stream>>>(p.rows, p.ld, p.n, p.d, p.batch_cols, cents, K,
                                                                       key_stride, keys, done, best);
            break;
        case kTrainCos:
            nearest_centroid_kernel<kTrainCos><<<grid, 256, 0, stream>>>(p.rows, p.ld, p.n, p.d, p.batch_cols, cents,
                                                                        K, key_stride, keys, done, best);
            break;
        default:
            nearest_centroid_kernel<kTrainDot><<<grid, 256, 0, stream>>>(p.rows, p.ld, p.n, p.d, p.batch_cols, cents,
                                                                        K, key_stride, keys, done, best);
            break;
    }
    launch_ok("nearest centroid kernel");
}

int metric_mode(int metric) {
    switch (metric) {
        case kMetricCos: return kTrainCos;
        case kMetricL2: return kTrainL2;
        case kMetricDot: return kTrainDot;
    }
    fail(ELIPS_B200_UNSUPPORTED_METRIC, "unknown metric");
}

void check_rows(const TrainRows& p, uint32_t K) {
    if (p.n == 0 || p.d == 0 || K == 0) fail(ELIPS_B200_INVALID_ARGUMENT, "empty training problem");
    if (p.n > 0xFFFFFFFFull || p.n * p.batch > 0xFFFFFFFFull)
        fail(ELIPS_B200_INVALID_ARGUMENT, "at most 2^32 - 1 (row, batch) pairs per training call");
    if (static_cast<uint64_t>(K) * p.batch > 0xFFFFFFFFull)
        fail(ELIPS_B200_INVALID_ARGUMENT, "too many centroids");
}

// Lloyd's k-means on the device. ivf = false: quant::detail::kmeans
// (squared L2, `iters` rounds, a batch stops once no centroid moved);
// ivf = true: IvfIndexState::train_centroids (metric distance, max(1, iters)
// rounds, cosine centroids normalised). cents: [batch][K][d].
void lloyd(const TrainRows& p, uint32_t K, size_t iters, bool ivf, int mode, float* cents, cudaStream_t stream) {
    check_rows(p, K);
    const uint64_t pairs = p.n * p.batch;
    const uint64_t keys_total = static_cast<uint64_t>(K) * p.batch;
    const uint64_t cent_total = keys_total * p.d;
    const uint64_t stride = std::max<uint64_t>(1, p.n / K);
    seed_centroids_kernel<<<blocks_for(cent_total, 256), 256, 0, stream>>>(p.rows, p.ld, p.n, p.d, p.batch_cols, K,
                                                                          cent_total, stride, cents);
    launch_ok("seed kernel");
    const size_t rounds = ivf ? std::max<size_t>(1, iters) : iters;
    if (rounds == 0) return;

    const int bits = key_bits(keys_total - 1);
    size_t temp = 0;
    check_cuda(cub::DeviceRadixSort::SortPairs(nullptr, temp, static_cast<const uint32_t*>(nullptr),
                                               static_cast<uint32_t*>(nullptr), static_cast<const uint32_t*>(nullptr),
                                               static_cast<uint32_t*>(nullptr), static_cast<int64_t>(pairs), 0, bits,
                                               stream),
               ELIPS_B200_KERNEL_LAUNCH_FAILED, "sort sizing");
    const size_t a_pairs = up256(pairs * 4), a_keys = up256(keys_total * 4), a_flags = up256(p.batch * 4ull);
    StreamScratch s(4 * a_pairs + 2 * a_keys + 2 * a_flags + up256(temp), stream);
    uint8_t* base = s.get();
    uint32_t* keys = reinterpret_cast<uint32_t*>(base);
    uint32_t* keys_sorted = reinterpret_cast<uint32_t*>(base + a_pairs);
    uint32_t* vals = reinterpret_cast<uint32_t*>(base + 2 * a_pairs);
    uint32_t* members = reinterpret_cast<uint32_t*>(base + 3 * a_pairs);
    uint32_t* start = reinterpret_cast<uint32_t*>(base + 4 * a_pairs);
    uint32_t* end = reinterpret_cast<uint32_t*>(base + 4 * a_pairs + a_keys);
    uint32_t* moved = reinterpret_cast<uint32_t*>(base + 4 * a_pairs + 2 * a_keys);
    uint32_t* done = reinterpret_cast<uint32_t*>(base + 4 * a_pairs + 2 * a_keys + a_flags);
    void* tmp = base + 4 * a_pairs + 2 * a_keys + 2 * a_flags;
    check_cuda(cudaMemsetAsync(moved, 0, 2 * a_flags, stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "flag reset");
    row_iota_kernel<<<blocks_for(pairs, 256), 256, 0, stream>>>(vals, p.n, pairs);
    launch_ok("iota kernel");
    const uint32_t* done_arg = ivf ? nullptr : done;
    std::vector<uint32_t> host_done(p.batch);
    for (size_t it = 0; it < rounds; ++it) {
        launch_nearest(mode, p, cents, K, K, keys, done_arg, stream);
        {
            Profiler::Scope prof("kmeans_sort", stream, pairs);
            check_cuda(cub::DeviceRadixSort::SortPairs(tmp, temp, keys, keys_sorted, vals, members,
                                                       static_cast<int64_t>(pairs), 0, bits, stream),
                       ELIPS_B200_KERNEL_LAUNCH_FAILED, "key sort");
        }
        check_cuda(cudaMemsetAsync(start, 0, 2 * a_keys, stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "bounds reset");
        segment_bounds_kernel<<<blocks_for(pairs, 256), 256, 0, stream>>>(keys_sorted, pairs, start, end);
        launch_ok("bounds kernel");
        {
            Profiler::Scope prof("centroid_update", stream, cent_total);
            if (ivf)
                centroid_update_kernel<true><<<blocks_for(cent_total, 256), 256, 0, stream>>>(
                    p.rows, p.ld, p.n, p.d, p.batch_cols, members, start, end, K, cent_total, cents, moved, nullptr);
            else
                centroid_update_kernel<false><<<blocks_for(cent_total, 256), 256, 0, stream>>>(
                    p.rows, p.ld, p.n, p.d, p.batch_cols, members, start, end, K, cent_total, cents, moved, done);
            launch_ok("update kernel");
        }
        if (ivf) {
            if (mode == kTrainCos) {
                centroid_normalize_kernel<<<blocks_for(K, 128), 128, 0, stream>>>(cents, K, p.d);
                launch_ok("normalize kernel");
            }
            continue;
        }
        kmeans_flags_kernel<<<blocks_for(p.batch, 128), 128, 0, stream>>>(moved, done, p.batch);
        launch_ok("flags kernel");
        check_cuda(cudaMemcpyAsync(host_done.data(), done, p.batch * 4ull, cudaMemcpyDeviceToHost, stream),
                   ELIPS_B200_TRANSFER_FAILED, "flag download");
        check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "k-means round");
        if (std::all_of(host_done.begin(), host_done.end(), [](uint32_t v) { return v != 0u; })) break;
    }
}

}  // namespace

void pq_encode_device(const float* rows, size_t n, size_t d, size_t m, size_t ksub, const float* codebook,
                      uint8_t* codes, cudaStream_t stream) {
    if (n == 0) return;
    if (m == 0 || d % m != 0 || m > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must divide by pq_dim");
    if (ksub == 0 || ksub > 256) fail(ELIPS_B200_INVALID_ARGUMENT, "ksub must be in [1, 256]");
    const uint32_t sub = static_cast<uint32_t>(d / m);
    const size_t chunk = std::max<size_t>(1, (size_t{1} << 26) / m);
    StreamScratch s(std::min(n, chunk) * m * 4, stream);
    uint32_t* keys = reinterpret_cast<uint32_t*>(s.get());
    for (size_t r0 = 0; r0 < n; r0 += chunk) {
        const size_t rows_here = std::min(chunk, n - r0);
        const TrainRows p{rows + r0 * d, d, rows_here, sub, static_cast<uint32_t>(m), sub};
        launch_nearest(kTrainSqL2, p, codebook, static_cast<uint32_t>(ksub), 0u, keys, nullptr, stream);
        const uint64_t total = static_cast<uint64_t>(rows_here) * m;
        keys_to_codes_kernel<<<blocks_for(total, 256), 256, 0, stream>>>(keys, rows_here, static_cast<uint32_t>(m),
                                                                        codes + r0 * m);
        launch_ok("code transpose kernel");
    }
}

void kmeans_device(int device, const float* rows, size_t n, size_t d, size_t k, size_t iters, float* cents,
                   cudaStream_t stream) {
    DeviceGuard g(device);
    device_props(device);
    if (d > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must be in [1, 65535]");
    const TrainRows p{rows, d, n, static_cast<uint32_t>(d), 1u, 0u};
    lloyd(p, static_cast<uint32_t>(k), iters, false, kTrainSqL2, cents, stream);
}

void train_pq_codebook_device(int device, const float* rows, size_t n, size_t d, size_t m, size_t ksub, size_t iters,
                              float* codebook, cudaStream_t stream) {
    DeviceGuard g(device);
    device_props(device);
    if (m == 0 || d == 0 || d % m != 0 || d > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must divide by pq_dim");
    if (ksub == 0 || ksub > 65536) fail(ELIPS_B200_INVALID_ARGUMENT, "ksub must be in [1, 65536]");
    const uint32_t sub = static_cast<uint32_t>(d / m);
    const TrainRows p{rows, d, n, sub, static_cast<uint32_t>(m), sub};
    lloyd(p, static_cast<uint32_t>(ksub), iters, false, kTrainSqL2, codebook, stream);
}

void ivf_assign_device(int device, int metric, const float* rows, size_t n, size_t d, const float* cents,
                       size_t n_lists, uint32_t* assign, float* dist, cudaStream_t stream) {
    if (n == 0) return;
    DeviceGuard g(device);
    device_props(device);
    const int mode = metric_mode(metric);
    if (d == 0 || d > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must be in [1, 65535]");
    const TrainRows p{rows, d, n, static_cast<uint32_t>(d), 1u, 0u};
    check_rows(p, static_cast<uint32_t>(n_lists));
    if (n_lists > 0xFFFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "too many lists");
    launch_nearest(mode, p, cents, static_cast<uint32_t>(n_lists), 0u, assign, nullptr, stream, dist);
}

void ivf_train_device(int device, int metric, const float* rows, size_t n, size_t d, size_t n_lists, size_t iters,
                      float* cents, uint32_t* assign, cudaStream_t stream) {
    DeviceGuard g(device);
    device_props(device);
    const int mode = metric_mode(metric);
    if (d == 0 || d > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must be in [1, 65535]");
    if (n_lists == 0 || n_lists > n) fail(ELIPS_B200_INVALID_ARGUMENT, "n_lists must be in [1, n]");
    const TrainRows p{rows, d, n, static_cast<uint32_t>(d), 1u, 0u};
    lloyd(p, static_cast<uint32_t>(n_lists), iters, true, mode, cents, stream);
    if (assign != nullptr) launch_nearest(mode, p, cents, static_cast<uint32_t>(n_lists), 0u, assign, nullptr, stream);
}

// GpuIVFPQIndex model build (GpuIVFPQIndex.cpp:88-131 after
// IvfIndexState::rebuild_from_current_data): centroids and assignments,
// residuals v - centroid, the PQ codebook trained on all residuals with 10
// rounds (GpuQuantizationPipeline.cpp:17-33), and the residual codes.
void ivfpq_train_device(int device, int metric, const float* rows, size_t n, size_t d, size_t n_lists, size_t iters,
                        size_t m, uint32_t pq_bits, float* cents, uint32_t* assign, float* codebook, uint8_t* codes,
                        cudaStream_t stream) {
    if (pq_bits < 1 || pq_bits > 8) fail(ELIPS_B200_INVALID_ARGUMENT, "pq_bits must be in [1, 8]");
    if (m == 0 || d % m != 0) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must divide by pq_dim");
    if (assign == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "assignments are required");
    ivf_train_device(device, metric, rows, n, d, n_lists, iters, cents, assign, stream);
    DeviceGuard g(device);
    const uint64_t total = static_cast<uint64_t>(n) * d;
    StreamScratch res(total * 4, stream);
    float* r = reinterpret_cast<float*>(res.get());
    residuals_kernel<<<blocks_for(total, 256), 256, 0, stream>>>(rows, assign, cents, n, static_cast<uint32_t>(d), r);
    launch_ok("residuals kernel");
    const size_t ksub = size_t{1} << pq_bits;
    train_pq_codebook_device(device, r, n, d, m, ksub, 10, codebook, stream);
    if (codes != nullptr) pq_encode_device(r, n, d, m, ksub, codebook, codes, stream);
}

}  // namespace eb

namespace {

using eb::guarded;
using eb::OwnedStream;

}  // namespace

extern "C" {

int elips_b200_kmeans(int device, const float* rows, size_t n, size_t dim, size_t k, size_t iters,
                      float* centroids_out, int pointers_on_device, void* stream) {
    if (rows == nullptr || centroids_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (n == 0 || dim == 0 || k == 0) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::kmeans_device(device, rows, n, dim, k, iters, centroids_out, static_cast<cudaStream_t>(stream));
            return;
        }
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            eb::StreamScratch s(eb::up256(n * dim * 4) + k * dim * 4, st.s);
            float* dr = reinterpret_cast<float*>(s.get());
            float* dc = reinterpret_cast<float*>(s.get() + eb::up256(n * dim * 4));
            eb::check_cuda(cudaMemcpyAsync(dr, rows, n * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row upload");
            eb::kmeans_device(device, dr, n, dim, k, iters, dc, st.s);
            eb::check_cuda(cudaMemcpyAsync(centroids_out, dc, k * dim * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "centroid download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "kmeans");
    });
}

int elips_b200_train_pq_codebook(int device, const float* rows, size_t n, size_t dim, size_t pq_dim, size_t ksub,
                                 size_t iters, float* codebook_out, int pointers_on_device, void* stream) {
    if (rows == nullptr || codebook_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (n == 0 || dim == 0 || pq_dim == 0 || dim % pq_dim != 0 || ksub == 0) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::train_pq_codebook_device(device, rows, n, dim, pq_dim, ksub, iters, codebook_out,
                                         static_cast<cudaStream_t>(stream));
            return;
        }
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            const size_t cb = ksub * dim * 4;
            eb::StreamScratch s(eb::up256(n * dim * 4) + cb, st.s);
            float* dr = reinterpret_cast<float*>(s.get());
            float* dc = reinterpret_cast<float*>(s.get() + eb::up256(n * dim * 4));
            eb::check_cuda(cudaMemcpyAsync(dr, rows, n * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row upload");
            eb::train_pq_codebook_device(device, dr, n, dim, pq_dim, ksub, iters, dc, st.s);
            eb::check_cuda(cudaMemcpyAsync(codebook_out, dc, cb, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "codebook download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "train_pq_codebook");
    });
}

int elips_b200_ivf_assign(int device, int metric, const float* rows, size_t n, size_t dim, const float* centroids,
                          size_t n_lists, uint32_t* assignments_out, float* distances_out, int pointers_on_device,
                          void* stream) {
    if (n > 0 && (rows == nullptr || centroids == nullptr || assignments_out == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    if (n > 0 && (dim == 0 || n_lists == 0)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::ivf_assign_device(device, metric, rows, n, dim, centroids, n_lists, assignments_out, distances_out,
                                  static_cast<cudaStream_t>(stream));
            return;
        }
        if (n == 0) return;
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            const size_t a_rows = eb::up256(n * dim * 4), a_cent = eb::up256(n_lists * dim * 4);
            const size_t a_asg = eb::up256(n * 4);
            eb::StreamScratch s(a_rows + a_cent + a_asg + n * 4, st.s);
            float* dr = reinterpret_cast<float*>(s.get());
            float* dc = reinterpret_cast<float*>(s.get() + a_rows);
            uint32_t* da = reinterpret_cast<uint32_t*>(s.get() + a_rows + a_cent);
            float* dd = reinterpret_cast<float*>(s.get() + a_rows + a_cent + a_asg);
            eb::check_cuda(cudaMemcpyAsync(dr, rows, n * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row upload");
            eb::check_cuda(cudaMemcpyAsync(dc, centroids, n_lists * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "centroid upload");
            eb::ivf_assign_device(device, metric, dr, n, dim, dc, n_lists, da, distances_out ? dd : nullptr, st.s);
            eb::check_cuda(cudaMemcpyAsync(assignments_out, da, n * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "assignment download");
            if (distances_out != nullptr)
                eb::check_cuda(cudaMemcpyAsync(distances_out, dd, n * 4, cudaMemcpyDeviceToHost, st.s),
                               ELIPS_B200_TRANSFER_FAILED, "distance download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "ivf_assign");
    });
}

int elips_b200_ivf_train(int device, int metric, const float* rows, size_t n, size_t dim, size_t n_lists,
                         size_t iters, float* centroids_out, uint32_t* assignments_out, int pointers_on_device,
                         void* stream) {
    if (rows == nullptr || centroids_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (n == 0 || dim == 0 || n_lists == 0 || n_lists > n) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::ivf_train_device(device, metric, rows, n, dim, n_lists, iters, centroids_out, assignments_out,
                                 static_cast<cudaStream_t>(stream));
            return;
        }
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            const size_t a_rows = eb::up256(n * dim * 4), a_cent = eb::up256(n_lists * dim * 4);
            eb::StreamScratch s(a_rows + a_cent + n * 4, st.s);
            float* dr = reinterpret_cast<float*>(s.get());
            float* dc = reinterpret_cast<float*>(s.get() + a_rows);
            uint32_t* da = reinterpret_cast<uint32_t*>(s.get() + a_rows + a_cent);
            eb::check_cuda(cudaMemcpyAsync(dr, rows, n * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row upload");
            eb::ivf_train_device(device, metric, dr, n, dim, n_lists, iters, dc,
                                 assignments_out != nullptr ? da : nullptr, st.s);
            eb::check_cuda(cudaMemcpyAsync(centroids_out, dc, n_lists * dim * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "centroid download");
            if (assignments_out != nullptr)
                eb::check_cuda(cudaMemcpyAsync(assignments_out, da, n * 4, cudaMemcpyDeviceToHost, st.s),
                               ELIPS_B200_TRANSFER_FAILED, "assignment download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "ivf_train");
    });
}

int elips_b200_ivfpq_train(int device, int metric, const float* rows, size_t n, size_t dim, size_t n_lists,
                           size_t iters, size_t pq_dim, uint32_t pq_bits, float* centroids_out,
                           uint32_t* assignments_out, float* codebook_out, uint8_t* codes_out, int pointers_on_device,
                           void* stream) {
    if (rows == nullptr || centroids_out == nullptr || assignments_out == nullptr || codebook_out == nullptr)
        return ELIPS_B200_INVALID_ARGUMENT;
    if (n == 0 || dim == 0 || n_lists == 0 || n_lists > n || pq_dim == 0 || dim % pq_dim != 0 || pq_bits < 1 ||
        pq_bits > 8)
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (pointers_on_device) {
            eb::ivfpq_train_device(device, metric, rows, n, dim, n_lists, iters, pq_dim, pq_bits, centroids_out,
                                   assignments_out, codebook_out, codes_out, static_cast<cudaStream_t>(stream));
            return;
        }
        eb::DeviceGuard g(device);
        OwnedStream st;
        {
            const size_t ksub = size_t{1} << pq_bits;
            const size_t a_rows = eb::up256(n * dim * 4), a_cent = eb::up256(n_lists * dim * 4);
            const size_t a_asg = eb::up256(n * 4), a_cb = eb::up256(ksub * dim * 4);
            eb::StreamScratch s(a_rows + a_cent + a_asg + a_cb + n * pq_dim, st.s);
            uint8_t* b = s.get();
            float* dr = reinterpret_cast<float*>(b);
            float* dc = reinterpret_cast<float*>(b + a_rows);
            uint32_t* da = reinterpret_cast<uint32_t*>(b + a_rows + a_cent);
            float* dcb = reinterpret_cast<float*>(b + a_rows + a_cent + a_asg);
            uint8_t* dcodes = b + a_rows + a_cent + a_asg + a_cb;
            eb::check_cuda(cudaMemcpyAsync(dr, rows, n * dim * 4, cudaMemcpyHostToDevice, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "row upload");
            eb::ivfpq_train_device(device, metric, dr, n, dim, n_lists, iters, pq_dim, pq_bits, dc, da, dcb,
                                   codes_out != nullptr ? dcodes : nullptr, st.s);
            eb::check_cuda(cudaMemcpyAsync(centroids_out, dc, n_lists * dim * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "centroid download");
            eb::check_cuda(cudaMemcpyAsync(assignments_out, da, n * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "assignment download");
            eb::check_cuda(cudaMemcpyAsync(codebook_out, dcb, ksub * dim * 4, cudaMemcpyDeviceToHost, st.s),
                           ELIPS_B200_TRANSFER_FAILED, "codebook download");
            if (codes_out != nullptr)
                eb::check_cuda(cudaMemcpyAsync(codes_out, dcodes, n * pq_dim, cudaMemcpyDeviceToHost, st.s),
                               ELIPS_B200_TRANSFER_FAILED, "code download");
        }
        eb::check_cuda(cudaStreamSynchronize(st.s), ELIPS_B200_KERNEL_LAUNCH_FAILED, "ivfpq_train");
    });
}

}  // extern "C"
