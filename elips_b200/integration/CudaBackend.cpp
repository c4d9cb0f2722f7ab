// elips::gpu::cuda::CudaBackend on the B200 library.
//
// ELIPS declares this class in src/gpu_engine/backends/cuda/CudaBackend.hpp:
// 12-56 (GpuPort, include/elips/gpu_engine/GpuPort.hpp:40-86) and ships its
// .cpp as an #error stub; GpuDeviceManager::probe_all_devices constructs it
// under ELIPS_CUDA_ENABLED (GpuDeviceManager.cpp:82-91). This file is that
// .cpp: every GpuPort call goes through the C ABI of libelips_b200.so
// (include/elips_b200.h), whose status codes 1..8 are GpuError + 1.
//
// Build (inside an ELIPS tree, or against one with -I): compile with
// -std=c++23 -DELIPS_CUDA_ENABLED -I<elips>/include -I<elips>/src/gpu_engine
// -I<this repo>/include, link libelips_b200.so and libcudart.
//
// Semantics kept from the port contract:
//  * compute_distances_batch / top_k take HOST spans (the callers in
//    GpuIVFPQIndex, GpuIVFFlatIndex, GpuSearchPipeline pass std::vector data);
//    the library copies them in and out on a stream of its own per call and
//    returns when the results are in host memory, so concurrent calls from
//    Vault::seek's reader threads are safe;
//  * results are bit-identical to the reference's scalar loops
//    (elips::distance sequential fp32, top_k ascending, ties by index);
//  * errors come back as std::expected, never as exceptions.
#include "backends/cuda/CudaBackend.hpp"

#include <string>

#include "elips_b200.h"

namespace elips::gpu::cuda {
namespace {

GpuError to_error(int status) {
    if (status >= ELIPS_B200_DEVICE_NOT_FOUND && status <= ELIPS_B200_BACKEND_UNAVAILABLE)
        return static_cast<GpuError>(status - 1);
    return GpuError::KernelLaunchFailed;  // dimension mismatch, bad argument, device timeout
}

std::expected<void, GpuError> to_expected(int status) {
    if (status == ELIPS_B200_OK) return {};
    return std::unexpected(to_error(status));
}

}  // namespace

CudaBackend::CudaBackend() = default;

CudaBackend::~CudaBackend() { shutdown(); }

std::expected<void, GpuError> CudaBackend::initialize(const GpuConfig& config) {
    if (initialized_) return {};
    int count = 0;
    if (elips_b200_device_count(&count) != ELIPS_B200_OK || count == 0)
        return std::unexpected(GpuError::DeviceNotFound);
    const int device = config.device_index < 0 ? 0 : config.device_index;
    if (device >= count) return std::unexpected(GpuError::DeviceNotFound);
    if (cudaSetDevice(device) != cudaSuccess) return std::unexpected(GpuError::InitializationFailed);
    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess)
        return std::unexpected(GpuError::InitializationFailed);
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return std::unexpected(GpuError::InitializationFailed);
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    info_ = GpuDeviceInfo{};
    info_.name = prop.name;
    info_.vendor = "NVIDIA";
    info_.backend = "cuda";
    info_.device_index = static_cast<uint32_t>(device);
    info_.total_device_memory_bytes = total_b;
    info_.free_device_memory_bytes = free_b;
    info_.supports_fp16 = true;
    info_.supports_bf16 = true;
    info_.supports_int8 = true;
    info_.compute_capability_major = static_cast<uint32_t>(prop.major);
    info_.compute_capability_minor = static_cast<uint32_t>(prop.minor);
    info_.max_threads_per_block = static_cast<uint32_t>(prop.maxThreadsPerBlock);
    info_.multiprocessor_count = static_cast<uint32_t>(prop.multiProcessorCount);
    info_.shared_memory_per_block_bytes = prop.sharedMemPerBlockOptin;
    info_.l2_cache_bytes = static_cast<size_t>(prop.l2CacheSize);
    info_.supports_ivf_pq = true;
    info_.supports_dynamic_batching = true;
    info_.supports_half_precision_search = true;
    device_index_ = device;
    initialized_ = true;
    return {};
}

void CudaBackend::shutdown() noexcept {
    if (stream_ != nullptr) {
        cudaStreamSynchronize(stream_);
        cudaStreamDestroy(stream_);
        stream_ = nullptr;
    }
    initialized_ = false;
}

GpuDeviceInfo CudaBackend::device_info() const noexcept { return info_; }

bool CudaBackend::is_available() const noexcept { return initialized_; }

std::expected<GpuBuffer, GpuError> CudaBackend::allocate_device(size_t bytes) {
    if (!initialized_) return std::unexpected(GpuError::BackendUnavailable);
    if (cudaSetDevice(device_index_) != cudaSuccess) return std::unexpected(GpuError::DeviceNotFound);
    void* ptr = nullptr;
    if (bytes > 0 && cudaMalloc(&ptr, bytes) != cudaSuccess) return std::unexpected(GpuError::InsufficientMemory);
    return GpuBuffer{ptr, bytes, this};
}

void CudaBackend::free_device(GpuBuffer buf) noexcept {
    if (buf.device_ptr() != nullptr) {
        cudaSetDevice(device_index_);
        cudaFree(buf.device_ptr());
    }
}

std::expected<void, GpuError> CudaBackend::upload(const void* host_src, GpuBuffer& dst, size_t bytes) {
    if (!initialized_) return std::unexpected(GpuError::BackendUnavailable);
    if (bytes > dst.bytes() || (bytes > 0 && (host_src == nullptr || dst.device_ptr() == nullptr)))
        return std::unexpected(GpuError::TransferFailed);
    if (bytes == 0) return {};
    cudaSetDevice(device_index_);
    if (cudaMemcpyAsync(dst.device_ptr(), host_src, bytes, cudaMemcpyHostToDevice, stream_) != cudaSuccess ||
        cudaStreamSynchronize(stream_) != cudaSuccess)
        return std::unexpected(GpuError::TransferFailed);
    return {};
}

std::expected<void, GpuError> CudaBackend::download(const GpuBuffer& src, void* host_dst, size_t bytes) {
    if (!initialized_) return std::unexpected(GpuError::BackendUnavailable);
    if (bytes > src.bytes() || (bytes > 0 && (host_dst == nullptr || src.device_ptr() == nullptr)))
        return std::unexpected(GpuError::TransferFailed);
    if (bytes == 0) return {};
    cudaSetDevice(device_index_);
    if (cudaMemcpyAsync(host_dst, src.device_ptr(), bytes, cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
        cudaStreamSynchronize(stream_) != cudaSuccess)
        return std::unexpected(GpuError::TransferFailed);
    return {};
}

std::expected<void, GpuError> CudaBackend::compute_distances_batch(std::span<const float> queries,
                                                                   std::span<const float> database,
                                                                   std::span<float> distances_out, size_t nq,
                                                                   size_t nb, size_t dim, elips::Metric metric) {
    if (!initialized_) return std::unexpected(GpuError::BackendUnavailable);
    if (queries.size() < nq * dim || database.size() < nb * dim || distances_out.size() < nq * nb)
        return std::unexpected(GpuError::KernelLaunchFailed);
    return to_expected(elips_b200_compute_distances_batch(device_index_, queries.data(), database.data(),
                                                          distances_out.data(), nq, nb, dim,
                                                          static_cast<int>(metric), 0, nullptr));
}

std::expected<void, GpuError> CudaBackend::top_k(std::span<const float> distances, std::span<uint32_t> indices_out,
                                                 std::span<float> values_out, size_t nq, size_t nb, size_t k) {
    if (!initialized_) return std::unexpected(GpuError::BackendUnavailable);
    if (distances.size() < nq * nb || indices_out.size() < nq * k || values_out.size() < nq * k)
        return std::unexpected(GpuError::KernelLaunchFailed);
    return to_expected(elips_b200_top_k(device_index_, distances.data(), indices_out.data(), values_out.data(), nq,
                                        nb, k, 0, nullptr));
}

// Row-major C[m][n] = op(A) op(B), op(A) is m x k_inner, op(B) k_inner x n
// (HOST spans), in fp32 through the library's GEMM kernel.
std::expected<void, GpuError> CudaBackend::gemm_fp32(std::span<const float> a, std::span<const float> b,
                                                     std::span<float> c, size_t m, size_t n, size_t k_inner,
                                                     bool trans_a, bool trans_b) {
    if (!initialized_) return std::unexpected(GpuError::BackendUnavailable);
    if (a.size() < m * k_inner || b.size() < k_inner * n || c.size() < m * n)
        return std::unexpected(GpuError::KernelLaunchFailed);
    return to_expected(elips_b200_gemm_fp32(device_index_, a.data(), b.data(), c.data(), m, n, k_inner,
                                            trans_a ? 1 : 0, trans_b ? 1 : 0, 0, nullptr));
}

void CudaBackend::synchronize() {
    if (stream_ != nullptr) cudaStreamSynchronize(stream_);
}

bool CudaBackend::is_idle() const noexcept { return stream_ == nullptr || cudaStreamQuery(stream_) == cudaSuccess; }

}  // namespace elips::gpu::cuda
