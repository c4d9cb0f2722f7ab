// extern "C" surface declared in include/elips_b200.h. Each function catches
// every C++ exception and returns a status code; nothing throws across it.
#include <cstdio>
#include <cstring>
#include <string>
#include <new>

#include "../../include/elips_b200.h"
#include "engine.cuh"
#include "capi_util.cuh"
#include "profiler.cuh"

struct elips_b200_exact {
    eb::ExactIndex index;
};

namespace {

using eb::guarded;

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

size_t mask_words(size_t n) { return (n + 31) / 32; }

}  // namespace

extern "C" {

const char* elips_b200_status_string(int status) {
    switch (status) {
        case ELIPS_B200_OK: return "Ok";
        case ELIPS_B200_DEVICE_NOT_FOUND: return "DeviceNotFound";
        case ELIPS_B200_INSUFFICIENT_MEMORY: return "InsufficientMemory";
        case ELIPS_B200_KERNEL_LAUNCH_FAILED: return "KernelLaunchFailed";
        case ELIPS_B200_TRANSFER_FAILED: return "TransferFailed";
        case ELIPS_B200_INDEX_BUILD_FAILED: return "IndexBuildFailed";
        case ELIPS_B200_UNSUPPORTED_METRIC: return "UnsupportedMetric";
        case ELIPS_B200_INITIALIZATION_FAILED: return "InitializationFailed";
        case ELIPS_B200_BACKEND_UNAVAILABLE: return "BackendUnavailable";
        case ELIPS_B200_DIMENSION_MISMATCH: return "DimensionMismatch";
        case ELIPS_B200_INVALID_ARGUMENT: return "InvalidArgument";
        case ELIPS_B200_DEVICE_TIMEOUT: return "DeviceTimeout";
        default: return "Unknown";
    }
}

int elips_b200_device_count(int* count_out) {
    if (count_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count_out = 0;
        return e == cudaErrorNoDevice ? ELIPS_B200_DEVICE_NOT_FOUND : ELIPS_B200_BACKEND_UNAVAILABLE;
    }
    *count_out = n;
    return ELIPS_B200_OK;
}

int elips_b200_device_error(int device, int* code_out) {
    if (code_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { *code_out = eb::read_and_clear_device_error(device); });
}

int elips_b200_wait_selftest(int device, uint64_t cycles) {
    int code = 0;
    const int st = guarded([&] { code = eb::wait_selftest(device, static_cast<long long>(cycles)); });
    if (st != ELIPS_B200_OK) return st;
    return code != 0 ? ELIPS_B200_DEVICE_TIMEOUT : ELIPS_B200_OK;
}

int elips_b200_exact_create(int device, int metric, int precision, uint32_t dimension,
                            elips_b200_exact** out) {
    if (out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *out = nullptr;
    return guarded([&] {
        *out = new elips_b200_exact{eb::ExactIndex(device, metric, precision, dimension)};
    });
}

int elips_b200_exact_add(elips_b200_exact* index, const void* rows, size_t n) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.add(rows, n); });
}

int elips_b200_exact_add_device(elips_b200_exact* index, const void* rows, size_t n, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.add_device(rows, n, as_stream(stream)); });
}

int elips_b200_exact_size(const elips_b200_exact* index, size_t* n_out) {
    if (index == nullptr || n_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *n_out = index->index.size();
    return ELIPS_B200_OK;
}

int elips_b200_exact_live(const elips_b200_exact* index, size_t* n_out) {
    if (index == nullptr || n_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *n_out = index->index.live();
    return ELIPS_B200_OK;
}

int elips_b200_exact_device_bytes(const elips_b200_exact* index, size_t* bytes_out) {
    if (index == nullptr || bytes_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *bytes_out = index->index.device_bytes();
    return ELIPS_B200_OK;
}

int elips_b200_exact_remove(elips_b200_exact* index, size_t row, int* removed_out) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        const bool r = index->index.remove(row);
        if (removed_out != nullptr) *removed_out = r ? 1 : 0;
    });
}

int elips_b200_exact_compact(elips_b200_exact* index, uint32_t* new_to_old, size_t capacity) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (new_to_old != nullptr && capacity < index->index.live()) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.compact(new_to_old); });
}

int elips_b200_exact_snapshot_bytes(const elips_b200_exact* index, size_t* bytes_out) {
    if (index == nullptr || bytes_out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *bytes_out = index->index.blob_bytes();
    return ELIPS_B200_OK;
}

int elips_b200_exact_export(const elips_b200_exact* index, void* out, size_t bytes) {
    if (index == nullptr || out == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.export_blob(out, bytes); });
}

int elips_b200_exact_import(elips_b200_exact* index, const void* blob, size_t bytes) {
    if (index == nullptr || blob == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] { index->index.import_blob(blob, bytes); });
}

int elips_b200_exact_destroy(elips_b200_exact* index) {
    if (index == nullptr) return ELIPS_B200_OK;
    return guarded([&] {
        eb::DeviceGuard g(index->index.device());
        delete index;
    });
}

int elips_b200_exact_search(const elips_b200_exact* index, const void* queries, size_t nq,
                            size_t k, const uint32_t* mask, float* out_dist, int64_t* out_rows) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (queries == nullptr || out_dist == nullptr || out_rows == nullptr))
        return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        const eb::ExactIndex& ix = index->index;
        if (nq == 0 || k == 0) return;
        eb::DeviceGuard g(ix.device());
        cudaStream_t stream = nullptr;
        eb::check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking),
                       ELIPS_B200_INITIALIZATION_FAILED, "cudaStreamCreate");
        struct StreamOwner {
            cudaStream_t s;
            ~StreamOwner() { cudaStreamDestroy(s); }
        } owner{stream};
        const size_t in_elem = ix.kind() == eb::OperandKind::I8 ? 1 : 4;
        const size_t q_bytes = nq * ix.dim() * in_elem;
        const size_t m_bytes = mask ? mask_words(ix.size()) * 4 : 0;
        const size_t o_bytes = nq * k * (sizeof(float) + sizeof(int64_t));
        {
            eb::StreamScratch io(q_bytes + m_bytes + o_bytes + 512, stream);
            uint8_t* base = io.get();
            void* dq = base;
            uint32_t* dm = mask ? reinterpret_cast<uint32_t*>(base + (q_bytes + 255) / 256 * 256) : nullptr;
            uint8_t* obase = base + (q_bytes + 255) / 256 * 256 + (m_bytes + 255) / 256 * 256;
            float* dd = reinterpret_cast<float*>(obase);
            int64_t* dr = reinterpret_cast<int64_t*>(obase + ((nq * k * sizeof(float) + 255) / 256 * 256));
            eb::check_cuda(cudaMemcpyAsync(dq, queries, q_bytes, cudaMemcpyHostToDevice, stream),
                           ELIPS_B200_TRANSFER_FAILED, "query upload");
            if (mask)
                eb::check_cuda(cudaMemcpyAsync(dm, mask, m_bytes, cudaMemcpyHostToDevice, stream),
                               ELIPS_B200_TRANSFER_FAILED, "mask upload");
            ix.search_device(dq, nq, k, dm, 0, dd, dr, nullptr, stream);
            eb::check_cuda(cudaMemcpyAsync(out_dist, dd, nq * k * sizeof(float), cudaMemcpyDeviceToHost, stream),
                           ELIPS_B200_TRANSFER_FAILED, "distance download");
            eb::check_cuda(cudaMemcpyAsync(out_rows, dr, nq * k * sizeof(int64_t), cudaMemcpyDeviceToHost, stream),
                           ELIPS_B200_TRANSFER_FAILED, "row download");
        }
        eb::check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "search");
        if (eb::read_and_clear_device_error(ix.device()) != 0)
            eb::fail(ELIPS_B200_DEVICE_TIMEOUT, "a device-side wait timed out");
    });
}

int elips_b200_exact_search_device(const elips_b200_exact* index, const void* queries,
                                   size_t nq, size_t k, const uint32_t* mask, float* out_dist,
                                   int64_t* out_rows, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (out_dist == nullptr || out_rows == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        index->index.search_device(queries, nq, k, mask, 0, out_dist, out_rows, nullptr, as_stream(stream));
    });
}

int elips_b200_exact_search_candidates_device(const elips_b200_exact* index,
                                              const void* queries, size_t nq, size_t k,
                                              const uint32_t* mask, uint32_t row_offset,
                                              uint32_t* out_cand, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && out_cand == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (static_cast<uint64_t>(row_offset) + index->index.size() >= 0xFFFFFFFFull)
            eb::fail(ELIPS_B200_INVALID_ARGUMENT, "row_offset + size exceeds the 32-bit row space");
        index->index.search_device(queries, nq, k, mask, row_offset, nullptr, nullptr,
                                   reinterpret_cast<uint2*>(out_cand), as_stream(stream));
    });
}

int elips_b200_exact_search_candidates_shared_device(const elips_b200_exact* index, const void* queries,
                                                     size_t nq, size_t k, const uint32_t* mask, uint32_t row_offset,
                                                     uint32_t* out_cand, uint32_t* shared_bound, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (out_cand == nullptr || shared_bound == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        if (static_cast<uint64_t>(row_offset) + index->index.size() >= 0xFFFFFFFFull)
            eb::fail(ELIPS_B200_INVALID_ARGUMENT, "row_offset + size exceeds the 32-bit row space");
        index->index.search_device(queries, nq, k, mask, row_offset, nullptr, nullptr,
                                   reinterpret_cast<uint2*>(out_cand), as_stream(stream), shared_bound);
    });
}

int elips_b200_peer_alloc(int device, size_t bytes, void** ptr_out, void* ipc_handle_out) {
    if (ptr_out == nullptr || ipc_handle_out == nullptr || bytes == 0) return ELIPS_B200_INVALID_ARGUMENT;
    *ptr_out = nullptr;
    return guarded([&] {
        eb::DeviceGuard g(device);
        void* p = nullptr;
        eb::check_cuda(cudaMalloc(&p, bytes), ELIPS_B200_INSUFFICIENT_MEMORY, "peer buffer");
        cudaIpcMemHandle_t h;
        const cudaError_t e = cudaIpcGetMemHandle(&h, p);
        if (e != cudaSuccess) {
            cudaFree(p);
            eb::fail(ELIPS_B200_INITIALIZATION_FAILED, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
        }
        std::memcpy(ipc_handle_out, &h, sizeof(h));
        *ptr_out = p;
    });
}

int elips_b200_peer_open(int device, const void* ipc_handle, void** ptr_out) {
    if (ptr_out == nullptr || ipc_handle == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *ptr_out = nullptr;
    return guarded([&] {
        eb::DeviceGuard g(device);
        cudaIpcMemHandle_t h;
        std::memcpy(&h, ipc_handle, sizeof(h));
        eb::check_cuda(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess),
                       ELIPS_B200_INITIALIZATION_FAILED, "cudaIpcOpenMemHandle");
    });
}

int elips_b200_peer_close(int device, void* ptr) {
    if (ptr == nullptr) return ELIPS_B200_OK;
    return guarded([&] {
        eb::DeviceGuard g(device);
        eb::check_cuda(cudaIpcCloseMemHandle(ptr), ELIPS_B200_INITIALIZATION_FAILED, "cudaIpcCloseMemHandle");
    });
}

int elips_b200_peer_free(int device, void* ptr) {
    if (ptr == nullptr) return ELIPS_B200_OK;
    return guarded([&] {
        eb::DeviceGuard g(device);
        eb::check_cuda(cudaFree(ptr), ELIPS_B200_INVALID_ARGUMENT, "peer buffer free");
    });
}

int elips_b200_copy_device(int device, void* dst, const void* src, size_t bytes, void* stream) {
    if (bytes == 0) return ELIPS_B200_OK;
    if (dst == nullptr || src == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        eb::DeviceGuard g(device);
        eb::check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, as_stream(stream)),
                       ELIPS_B200_TRANSFER_FAILED, "device copy");
    });
}

int elips_b200_fill_device(int device, void* dst, int byte_value, size_t bytes, void* stream) {
    if (bytes == 0) return ELIPS_B200_OK;
    if (dst == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        eb::DeviceGuard g(device);
        eb::check_cuda(cudaMemsetAsync(dst, byte_value, bytes, as_stream(stream)), ELIPS_B200_KERNEL_LAUNCH_FAILED,
                       "device fill");
    });
}

int elips_b200_merge_candidates_device(int device, const uint32_t* cand, size_t nq,
                                       size_t lists, size_t k, int metric, float* out_dist,
                                       int64_t* out_rows, void* stream) {
    if (metric < 0 || metric > 2) return ELIPS_B200_UNSUPPORTED_METRIC;
    if (nq > 0 && k > 0 && (out_dist == nullptr || out_rows == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && lists > 0 && cand == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0xFFFFFFFFull || lists * k > 0xFFFFFFFFull) return ELIPS_B200_INVALID_ARGUMENT;
    return guarded([&] {
        eb::DeviceGuard g(device);
        eb::device_props(device);
        eb::merge_candidates(device, reinterpret_cast<const uint2*>(cand), static_cast<uint32_t>(nq),
                             static_cast<uint32_t>(lists), static_cast<uint32_t>(k), k,
                             static_cast<uint64_t>(nq) * k, metric, out_dist, out_rows, nullptr,
                             as_stream(stream));
    });
}

int elips_b200_profiler_enable(int enabled) {
    eb::Profiler::get().set_enabled(enabled != 0);
    return ELIPS_B200_OK;
}

int elips_b200_profiler_stats(const char* kernel, uint64_t* launches, double* total_ms, uint64_t* items) {
    return guarded([&] {
        const eb::KernelStats s = eb::Profiler::get().query(kernel);
        if (launches) *launches = s.launches;
        if (total_ms) *total_ms = s.total_ms;
        if (items) *items = s.items;
    });
}

int elips_b200_profiler_reset(void) {
    return guarded([&] { eb::Profiler::get().reset(); });
}

int elips_b200_launch_count(uint64_t* launches) {
    if (launches == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    *launches = eb::Profiler::get().total_launches();
    return ELIPS_B200_OK;
}

}  // extern "C"
