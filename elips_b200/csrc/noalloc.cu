// Exact search that performs no device allocation.
//
// Some callers cannot call cudaMalloc (or cudaMallocAsync) at search time:
// a process whose device memory is already fully reserved by another
// allocator (a serving framework that pre-allocates its caching pool leaves
// nothing for a second allocator to take), and latency-critical request paths
// where an allocation can synchronise the device or stall behind another
// stream. For them, elips_b200_exact_search_noalloc runs the same fused search
// with its scratch taken from the fixed device array below.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds its kNoAllocScratchBytes until the process exits. In host
// code its name is only a host-side stand-in, so its device address is looked
// up once per device with cudaGetSymbolAddress (with that device current) and
// that address is what the kernels receive.
#include <array>
#include <cstdio>
#include <mutex>

#include "../../include/elips_b200.h"
#include "engine.cuh"

namespace {

// 64 MiB per device: fixed upper bound of one no-alloc call's scratch.
constexpr size_t kNoAllocScratchBytes = size_t{64} << 20;
// CTA cap for no-alloc calls: bounds the per-CTA candidate lists that the
// scratch has to hold (2 x 128 lists of up to 512 entries per CTA).
constexpr uint32_t kNoAllocMaxGrid = 32;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
std::array<uint8_t*, kMaxDevices> g_noalloc_ptr{};

// Device address of the scratch array on `device` (looked up on first use,
// with the device current). Looking it up allocates nothing.
uint8_t* noalloc_scratch(int device) {
    if (device < 0 || device >= kMaxDevices) eb::fail(ELIPS_B200_DEVICE_NOT_FOUND, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[device] == nullptr) {
        eb::DeviceGuard g(device);
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr)
            eb::fail(ELIPS_B200_INITIALIZATION_FAILED,
                     std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
        g_noalloc_ptr[device] = static_cast<uint8_t*>(ptr);
    }
    return g_noalloc_ptr[device];
}

}  // namespace

struct elips_b200_exact {
    eb::ExactIndex index;
};

extern "C" int elips_b200_exact_search_noalloc(const elips_b200_exact* index, const void* queries,
                                               size_t nq, size_t k, const uint32_t* mask,
                                               float* out_dist, int64_t* out_rows, void* stream) {
    if (index == nullptr) return ELIPS_B200_INVALID_ARGUMENT;
    if (nq > 0 && k > 0 && (out_dist == nullptr || out_rows == nullptr)) return ELIPS_B200_INVALID_ARGUMENT;
    try {
        const eb::ExactIndex& ix = index->index;
        uint8_t* scratch = noalloc_scratch(ix.device());
        ix.search_device_in_scratch(queries, nq, k, mask, out_dist, out_rows, scratch, kNoAllocScratchBytes,
                                    kNoAllocMaxGrid, static_cast<cudaStream_t>(stream));
        return ELIPS_B200_OK;
    } catch (const eb::Error& e) {
        std::fprintf(stderr, "elips_b200: %s\n", e.what.c_str());
        return e.code;
    } catch (...) {
        return ELIPS_B200_KERNEL_LAUNCH_FAILED;
    }
}
