// Host engine for the exact search path: device set-up, buffers, TMA
// descriptors, launch planning, and the ExactIndex implementation.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "../../include/elips_b200.h"
#include "aux_kernels.cuh"
#include "engine.cuh"
#include "exact_topk.cuh"
#include "profiler.cuh"

namespace eb {

void fail(int code, const std::string& what) { throw Error{code, what}; }

void check_cuda(cudaError_t e, int code, const char* what) {
    if (e == cudaSuccess) return;
    if (e == cudaErrorMemoryAllocation) code = ELIPS_B200_INSUFFICIENT_MEMORY;
    fail(code, std::string(what) + ": " + cudaGetErrorString(e));
}

DeviceGuard::DeviceGuard(int device) {
    check_cuda(cudaGetDevice(&prev_), ELIPS_B200_DEVICE_NOT_FOUND, "cudaGetDevice");
    if (prev_ != device) check_cuda(cudaSetDevice(device), ELIPS_B200_DEVICE_NOT_FOUND, "cudaSetDevice");
}

DeviceGuard::~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev_ && prev_ >= 0) cudaSetDevice(prev_);
}

namespace {

std::mutex g_props_mu;
std::vector<DeviceProps> g_props;
std::vector<bool> g_props_ready;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    std::lock_guard<std::mutex> lock(g_props_mu);
    if (g_encode == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
                   ELIPS_B200_INITIALIZATION_FAILED, "cudaGetDriverEntryPoint");
        if (fn == nullptr || q != cudaDriverEntryPointSuccess)
            fail(ELIPS_B200_INITIALIZATION_FAILED, "cuTensorMapEncodeTiled unavailable");
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return g_encode;
}

}  // namespace

const DeviceProps& device_props(int device) {
    std::lock_guard<std::mutex> lock(g_props_mu);
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
        fail(ELIPS_B200_DEVICE_NOT_FOUND, "no such CUDA device");
    if (g_props.size() < static_cast<size_t>(count)) {
        g_props.resize(count);
        g_props_ready.resize(count, false);
    }
    if (!g_props_ready[device]) {
        cudaDeviceProp prop{};
        check_cuda(cudaGetDeviceProperties(&prop, device), ELIPS_B200_DEVICE_NOT_FOUND,
                   "cudaGetDeviceProperties");
        if (prop.major != 10 || prop.minor != 0)
            fail(ELIPS_B200_BACKEND_UNAVAILABLE, "device is not sm_100 (B200)");
        DeviceProps p;
        p.num_sms = prop.multiProcessorCount;
        p.cc_major = prop.major;
        p.cc_minor = prop.minor;
        p.max_smem_optin = prop.sharedMemPerBlockOptin;
        // Keep freed stream-ordered scratch cached in the pool between calls.
        cudaMemPool_t pool;
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
            uint64_t threshold = UINT64_MAX;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
        }
        if (prev >= 0) cudaSetDevice(prev);
        g_props[device] = p;
        g_props_ready[device] = true;
    }
    return g_props[device];
}

DeviceBuffer::DeviceBuffer(int device, size_t bytes) : device_(device), bytes_(bytes) {
    if (bytes == 0) return;
    DeviceGuard g(device);
    check_cuda(cudaMalloc(&ptr_, bytes), ELIPS_B200_INSUFFICIENT_MEMORY, "cudaMalloc");
}

DeviceBuffer::~DeviceBuffer() { reset(); }

DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
        reset();
        device_ = o.device_;
        ptr_ = o.ptr_;
        bytes_ = o.bytes_;
        o.ptr_ = nullptr;
        o.bytes_ = 0;
    }
    return *this;
}

void DeviceBuffer::reset() {
    if (ptr_ != nullptr) {
        int prev = -1;
        cudaGetDevice(&prev);
        if (prev != device_) cudaSetDevice(device_);
        cudaFree(ptr_);
        if (prev != device_ && prev >= 0) cudaSetDevice(prev);
    }
    ptr_ = nullptr;
    bytes_ = 0;
}

StreamScratch::StreamScratch(size_t bytes, cudaStream_t stream) : stream_(stream) {
    check_cuda(cudaMallocAsync(&ptr_, std::max<size_t>(bytes, 256), stream),
               ELIPS_B200_INSUFFICIENT_MEMORY, "cudaMallocAsync");
}

StreamScratch::~StreamScratch() {
    if (ptr_ != nullptr) cudaFreeAsync(ptr_, stream_);
}

void allow_dynamic_smem(const void* func, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, size_t> granted;
    int device = 0;
    check_cuda(cudaGetDevice(&device), ELIPS_B200_DEVICE_NOT_FOUND, "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    size_t& cur = granted[{device, func}];
    if (bytes <= cur) return;
    check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
               ELIPS_B200_KERNEL_LAUNCH_FAILED, "cudaFuncSetAttribute");
    cur = bytes;
}

CUtensorMap make_operand_map(const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                             uint64_t cols, uint64_t rows, uint32_t box_rows) {
    CUtensorMap map;
    std::memset(&map, 0, sizeof(map));
    const cuuint64_t dims[2] = {cols, std::max<uint64_t>(rows, 1)};
    const cuuint64_t strides[1] = {cols * elem_bytes};
    const cuuint32_t box[2] = {128u / elem_bytes, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(
        &map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(ELIPS_B200_KERNEL_LAUNCH_FAILED, "cuTensorMapEncodeTiled failed");
    return map;
}

ExactPlan plan_exact(uint32_t nq, uint32_t n, uint32_t k, uint32_t bn, int groups, uint32_t cg) {
    ExactPlan p;
    p.bn = bn;
    p.cg = cg;
    const int num_sms = groups;
    p.n_qt = (nq + kTileM * cg - 1) / (kTileM * cg);
    p.n_bt = (n + bn - 1) / bn;
    // Pick the smallest number of base splits whose (query tile, split)
    // units fill the SMs in whole waves; each split keeps >= 4 base tiles.
    uint32_t best_s = 1;
    double best_eff = -1.0;
    const uint32_t max_s = std::max<uint32_t>(1, std::min<uint32_t>(256, p.n_bt / 4));
    for (uint32_t s = 1; s <= max_s; ++s) {
        const uint64_t units = static_cast<uint64_t>(p.n_qt) * s;
        const uint64_t waves = (units + num_sms - 1) / num_sms;
        const double eff = static_cast<double>(units) / static_cast<double>(waves * num_sms);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best_s = s;
        }
        if (eff >= 0.97) break;
    }
    p.splits = best_s;
    const uint64_t units = static_cast<uint64_t>(p.n_qt) * p.splits;
    p.grid = static_cast<uint32_t>(std::min<uint64_t>(units, static_cast<uint64_t>(num_sms))) * cg;
    // List capacity: k survivors plus at least one whole half-tile of
    // admissions (compaction is checked once per tile); lists up to 512
    // entries are compacted in registers. Batches of one query tile run in a
    // single wave with no bound published yet, so their lists get a smaller
    // floor and compact (and tighten their own threshold) sooner.
    const uint32_t floor_cap = (cg == 1 && p.n_qt == 1) ? 256u : 512u;
    p.cap = std::max<uint32_t>(floor_cap, (k + bn / 2 + 32u + 31u) / 32u * 32u);
    return p;
}

// Entries each (query, split, column half) list publishes. In a batch of
// one query tile (8 to 128 queries) whose splits are at most 8 base tiles
// long, compacting every list to k at the end of its unit (one list at a
// time per warp) costs more than the unit's distances; there a list of up
// to 2k entries (rounded up to 32) is published as it is and the merge,
// which reads every list anyway, selects the k best. Otherwise k: longer
// units compact rarely at their end, and the merge would read padding.
// Measured on 100,000 x 384 bf16 L2, k = 20, per call: 64 queries 293 ->
// 208 us, 8 queries 112 -> 102 us; at 1,000,000 rows (26 tiles per split)
// 2k slots were 2-8 us slower, at one query 5 us slower.
// Entries after which a list compacts for the first time in a unit (0:
// only when it could overflow). For k <= 32 a list compacted at
// max(64, 2k) entries gets a threshold near its final one within the first
// tiles of a unit, where waiting until it nears its 512-entry capacity lets
// hundreds of candidates through: 100k x 128 fp32, 1,000 queries, k=10,
// 0.46 -> 0.37 ms per kernel, identical results. Larger k gained at most 2 %
// (250k x 768 fp16, k=100) and lost 3-9 % (5M x 1,024 int8, k=50); batches
// of one query tile, whose units are a few tiles long and publish their lists
// uncompacted, lost 40 %.
uint32_t early_compaction(uint32_t k, const ExactPlan& p) {
    if (k > 32u || (p.n_qt == 1 && p.cg == 1)) return 0u;
    return std::max<uint32_t>(64u, (2u * k + 31u) / 32u * 32u);
}

uint32_t publish_slot(const ExactPlan& p, uint32_t nq, uint32_t k) {
    if (p.n_qt != 1 || p.cg != 1 || nq < 8 || p.n_bt > 8u * p.splits) return k;
    return std::min<uint32_t>(p.cap, (2u * k + 31u) / 32u * 32u);
}

namespace {

constexpr uint32_t kMaxK = 1024;
// Bases smaller than this are searched whole even when a row filter is given.
constexpr size_t kGatherMinRows = 65536;

uint32_t elem_bytes_of(OperandKind k) {
    switch (k) {
        case OperandKind::F16:
        case OperandKind::BF16: return 2;
        case OperandKind::TF32X3: return 4;
        case OperandKind::I8: return 1;
    }
    return 2;
}

CUtensorMapDataType tma_dtype_of(OperandKind k) {
    switch (k) {
        case OperandKind::F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        case OperandKind::BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        case OperandKind::TF32X3: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        case OperandKind::I8: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
    }
    return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// Converts `rows` device rows (fp32 or int8) into operand layout at `dst_row`.
void prep_operands(OperandKind kind, const void* src, size_t rows, uint32_t dim, uint32_t d_pad,
                   void* ops, void* ops_lo, float* norms, cudaStream_t stream) {
    if (rows == 0) return;
    if (kind == OperandKind::I8) {
        const uint64_t total = static_cast<uint64_t>(rows) * d_pad;
        const uint32_t blocks = static_cast<uint32_t>((total + 255) / 256);
        Profiler::Scope prof("prep_rows", stream, rows);
        prep_rows_i8_kernel<<<blocks, 256, 0, stream>>>(static_cast<const int8_t*>(src), rows, dim,
                                                        d_pad, static_cast<int8_t*>(ops));
    } else {
        const int k = kind == OperandKind::F16 ? 0 : (kind == OperandKind::BF16 ? 1 : 2);
        const uint64_t threads = static_cast<uint64_t>(rows) * 32;
        const uint32_t blocks = static_cast<uint32_t>((threads + 255) / 256);
        Profiler::Scope prof("prep_rows", stream, rows);
        prep_rows_f32_kernel<<<blocks, 256, 0, stream>>>(static_cast<const float*>(src), rows, dim,
                                                         d_pad, k, ops, static_cast<float*>(ops_lo),
                                                         norms);
    }
    check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "prep kernel launch");
}

// Launch configuration of one exact kernel instantiation; CTA pairs are
// launched as clusters of two.
template <OperandKind KIND, int BN, int STAGES, int METRIC, int CG>
cudaLaunchConfig_t exact_launch_config(uint32_t grid, cudaStream_t stream, cudaLaunchAttribute* attr) {
    using Cfg = ExactConfig<KIND, BN, STAGES, CG>;
    auto kernel = exact_topk_kernel<KIND, BN, STAGES, METRIC, CG>;
    allow_dynamic_smem(reinterpret_cast<const void*>(kernel), Cfg::kSmemBytes);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kExactThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CG == 2 ? 1 : 0;
    return cfg;
}

template <OperandKind KIND, int BN, int STAGES, int METRIC, int CG>
void launch_exact_kernel(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& alo,
                         const CUtensorMap& blo, const ExactParams& params, uint32_t grid,
                         cudaStream_t stream) {
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = exact_launch_config<KIND, BN, STAGES, METRIC, CG>(grid, stream, attr);
    Profiler::Scope prof("exact_topk", stream, static_cast<uint64_t>(params.nq) * params.n);
    check_cuda(cudaLaunchKernelEx(&cfg, exact_topk_kernel<KIND, BN, STAGES, METRIC, CG>, a, b, alo, blo, params),
               ELIPS_B200_KERNEL_LAUNCH_FAILED, "exact kernel launch");
}

uint32_t bn_of(OperandKind k) { return k == OperandKind::TF32X3 ? 128u : 256u; }

// Candidates per query that the merge kernel keeps in shared memory.
constexpr uint64_t kMergeCacheMax = 2048;

// Lists merged per first-stage warp of a two-stage merge, or `lists` (one
// stage). Two stages when a batch has too few queries to give every SM work
// with one warp per query, or when a query's candidates do not fit the merge
// kernel's shared-memory cache. Groups hold up to 16 lists and, where the
// list length allows, at most 2048 / len so each group is merged from the cache (at least
// 8 lists for small batches, at least 2 otherwise); the last group takes the
// remainder.
uint32_t merge_group_size(uint32_t nq, uint32_t lists, uint32_t len, int num_sms) {
    const bool few_queries = nq < 8u * static_cast<uint32_t>(num_sms) && lists >= 8;
    const bool uncached = static_cast<uint64_t>(lists) * len > kMergeCacheMax && lists >= 4;
    if (!few_queries && !uncached) return lists;
    const uint32_t fit = static_cast<uint32_t>(kMergeCacheMax / std::max<uint32_t>(1u, len));
    const uint32_t g = std::min<uint32_t>(16u, std::max<uint32_t>(few_queries ? 8u : 2u, fit));
    return g < lists ? g : lists;
}

// The per-split candidate lists of every query merged into its k best. With
// groups == 0 in one pass. Otherwise (few queries, where one warp per query
// would walk all lists alone, or more candidates per query than the merge
// cache holds) every group of merge_group lists is first reduced to its k
// best, one warp per (query, group), into `stage`, then the groups are
// merged: the k smallest (key, row) of the k smallest of each group are the k
// smallest overall.
void merge_split_lists(int device, const uint2* part, uint2* stage, uint32_t nq, uint32_t n_lists,
                       uint32_t merge_group, uint32_t groups, uint32_t k, int metric, float* out_dist,
                       int64_t* out_rows, uint2* out_cand, cudaStream_t stream, uint32_t len) {
    if (groups > 0) {
        merge_candidates(device, part, nq, merge_group, k, static_cast<uint64_t>(n_lists) * len, len, metric, nullptr,
                         nullptr, stage, stream, groups, n_lists - (groups - 1) * merge_group, len);
        merge_candidates(device, stage, nq, groups, k, static_cast<uint64_t>(groups) * k, k, metric, out_dist,
                         out_rows, out_cand, stream);
        return;
    }
    merge_candidates(device, part, nq, n_lists, k, static_cast<uint64_t>(n_lists) * len, len, metric, out_dist,
                     out_rows, out_cand, stream, 1, 0, len);
}

// Pipeline depth: the stages that fit 192 KB of shared memory.
constexpr int stages_of(OperandKind k, int cg) {
    return k == OperandKind::TF32X3 ? (cg == 2 ? 4 : 3) : (cg == 2 ? 6 : 4);
}

template <OperandKind KIND, int BN, int CG>
void dispatch_metric(int metric, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& alo,
                     const CUtensorMap& blo, const ExactParams& prm, uint32_t grid, cudaStream_t stream) {
    constexpr int S = stages_of(KIND, CG);
    if constexpr (KIND == OperandKind::I8) {
        launch_exact_kernel<KIND, BN, S, kDot, CG>(a, b, alo, blo, prm, grid, stream);
    } else {
        switch (metric) {
            case kCosine: launch_exact_kernel<KIND, BN, S, kCosine, CG>(a, b, alo, blo, prm, grid, stream); break;
            case kEuclidean: launch_exact_kernel<KIND, BN, S, kEuclidean, CG>(a, b, alo, blo, prm, grid, stream); break;
            default: launch_exact_kernel<KIND, BN, S, kDot, CG>(a, b, alo, blo, prm, grid, stream); break;
        }
    }
}

template <int CG>
void dispatch_kind(OperandKind kind, int metric, const CUtensorMap& a, const CUtensorMap& b,
                   const CUtensorMap& alo, const CUtensorMap& blo, const ExactParams& prm, uint32_t grid,
                   cudaStream_t stream) {
    switch (kind) {
        case OperandKind::F16: dispatch_metric<OperandKind::F16, 256, CG>(metric, a, b, alo, blo, prm, grid, stream); break;
        case OperandKind::BF16: dispatch_metric<OperandKind::BF16, 256, CG>(metric, a, b, alo, blo, prm, grid, stream); break;
        case OperandKind::TF32X3: dispatch_metric<OperandKind::TF32X3, 128, CG>(metric, a, b, alo, blo, prm, grid, stream); break;
        case OperandKind::I8: dispatch_metric<OperandKind::I8, 256, CG>(metric, a, b, alo, blo, prm, grid, stream); break;
    }
}

void dispatch_exact(OperandKind kind, int metric, const CUtensorMap& a, const CUtensorMap& b,
                    const CUtensorMap& alo, const CUtensorMap& blo, const ExactParams& prm, const ExactPlan& plan,
                    cudaStream_t stream) {
    if (plan.cg == 2) dispatch_kind<2>(kind, metric, a, b, alo, blo, prm, plan.grid, stream);
    else dispatch_kind<1>(kind, metric, a, b, alo, blo, prm, plan.grid, stream);
}

// CTA pairs that can be resident at once (cluster occupancy of the pair
// kernel: 1 CTA per SM, two SMs of one GPC per pair), cached per device.
int pair_groups(int device) {
    static std::mutex mu;
    static int cached[64] = {0};
    std::lock_guard<std::mutex> lock(mu);
    if (device >= 0 && device < 64 && cached[device] > 0) return cached[device];
    const DeviceProps& props = device_props(device);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg =
        exact_launch_config<OperandKind::F16, 256, stages_of(OperandKind::F16, 2), kCosine, 2>(
            static_cast<uint32_t>(props.num_sms / 2 * 2), nullptr, attr);
    int clusters = 0;
    check_cuda(cudaOccupancyMaxActiveClusters(&clusters, exact_topk_kernel<OperandKind::F16, 256,
                                                                           stages_of(OperandKind::F16, 2), kCosine, 2>,
                                              &cfg),
               ELIPS_B200_KERNEL_LAUNCH_FAILED, "cluster occupancy");
    if (clusters <= 0) fail(ELIPS_B200_KERNEL_LAUNCH_FAILED, "no CTA pair fits on this device");
    if (device >= 0 && device < 64) cached[device] = clusters;
    return clusters;
}

}  // namespace

// The k <= 256 smallest (value, index) of every row of a distance matrix,
// one warp per row (topk_rows_warp_kernel).
void top_k_rows_warp(int device, const float* dist, uint32_t* idx, float* val, size_t nq, size_t nb, size_t k,
                     cudaStream_t stream) {
    constexpr uint32_t kWarps = 8;
    uint32_t kpow2 = 32;
    while (kpow2 < k) kpow2 <<= 1;
    const size_t smem = kWarps * (1024 + static_cast<size_t>(kpow2) * 8);
    allow_dynamic_smem(reinterpret_cast<const void*>(topk_rows_warp_kernel), smem);
    Profiler::Scope prof("topk_rows", stream, static_cast<uint64_t>(nq) * nb);
    const uint32_t blocks = static_cast<uint32_t>((nq + kWarps - 1) / kWarps);
    topk_rows_warp_kernel<<<blocks, kWarps * 32, smem, stream>>>(dist, static_cast<uint32_t>(nq),
                                                                  static_cast<uint32_t>(nb), static_cast<uint32_t>(k),
                                                                  kpow2, idx, val);
    check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "top-k rows launch");
    (void)device;
}

ExactIndex::ExactIndex(int device, int metric, int precision, uint32_t dim)
    : device_(device), metric_(metric), precision_(precision), dim_(dim) {
    if (dim == 0 || dim > 65535) fail(ELIPS_B200_INVALID_ARGUMENT, "dimension must be in [1, 65535]");
    if (metric < 0 || metric > 2) fail(ELIPS_B200_UNSUPPORTED_METRIC, "unknown metric");
    switch (precision) {
        case ELIPS_B200_PRECISION_FP32: kind_ = OperandKind::TF32X3; break;
        case ELIPS_B200_PRECISION_FP16:
        case ELIPS_B200_PRECISION_AUTO: kind_ = OperandKind::F16; break;
        case ELIPS_B200_PRECISION_BF16: kind_ = OperandKind::BF16; break;
        case ELIPS_B200_PRECISION_INT8: kind_ = OperandKind::I8; break;
        default: fail(ELIPS_B200_INVALID_ARGUMENT, "unknown precision");
    }
    if (kind_ == OperandKind::I8 && metric != kDot)
        fail(ELIPS_B200_UNSUPPORTED_METRIC, "the int8 codec scores inner product only");
    device_props(device);
    elem_bytes_ = elem_bytes_of(kind_);
    const uint32_t per_block = 128u / elem_bytes_;
    d_pad_ = (dim + per_block - 1) / per_block * per_block;
}

void ExactIndex::reserve(size_t rows) {
    if (rows <= capacity_) return;
    const size_t cap = std::max<size_t>(rows, capacity_ + capacity_ / 2);
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    DeviceBuffer ops(device_, cap * row_bytes);
    DeviceBuffer lo(device_, kind_ == OperandKind::TF32X3 ? cap * row_bytes : 0);
    DeviceBuffer norms(device_, metric_ == kEuclidean ? cap * sizeof(float) : 0);
    if (n_ > 0) {
        check_cuda(cudaMemcpy(ops.get(), ops_.get(), n_ * row_bytes, cudaMemcpyDeviceToDevice),
                   ELIPS_B200_TRANSFER_FAILED, "grow copy");
        if (lo.get() != nullptr)
            check_cuda(cudaMemcpy(lo.get(), ops_lo_.get(), n_ * row_bytes, cudaMemcpyDeviceToDevice),
                       ELIPS_B200_TRANSFER_FAILED, "grow copy");
        if (norms.get() != nullptr)
            check_cuda(cudaMemcpy(norms.get(), norms_.get(), n_ * sizeof(float), cudaMemcpyDeviceToDevice),
                       ELIPS_B200_TRANSFER_FAILED, "grow copy");
    }
    ops_ = std::move(ops);
    ops_lo_ = std::move(lo);
    norms_ = std::move(norms);
    capacity_ = cap;
    if (live_.get() != nullptr) {
        DeviceBuffer live(device_, (cap + 31) / 32 * 4);
        check_cuda(cudaMemcpy(live.get(), live_.get(), live_host_.size() * 4, cudaMemcpyDeviceToDevice),
                   ELIPS_B200_TRANSFER_FAILED, "grow copy");
        live_ = std::move(live);
    }
}

void ExactIndex::upload_live_words(size_t w0, size_t w1) {
    if (live_.get() == nullptr || w1 <= w0) return;
    check_cuda(cudaMemcpy(static_cast<uint32_t*>(live_.get()) + w0, live_host_.data() + w0, (w1 - w0) * 4,
                          cudaMemcpyHostToDevice),
               ELIPS_B200_TRANSFER_FAILED, "removal bits upload");
}

// Rows [first, first + count) become live (called for appended rows).
void ExactIndex::mark_live(size_t first, size_t count) {
    if (live_.get() == nullptr || count == 0) return;
    live_host_.resize((first + count + 31) / 32, 0u);
    for (size_t r = first; r < first + count; ++r) live_host_[r >> 5] |= 1u << (r & 31);
    upload_live_words(first >> 5, live_host_.size());
}

namespace {

// dst row i = src row idx[i], rows of `row_bytes` (a multiple of 16) bytes.
__global__ void gather_row_bytes_kernel(const uint4* __restrict__ src, const uint32_t* __restrict__ idx,
                                        uint64_t rows, uint32_t row_words, uint4* __restrict__ dst) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= rows * row_words) return;
    const uint64_t r = t / row_words;
    const uint32_t w = static_cast<uint32_t>(t % row_words);
    dst[t] = src[static_cast<uint64_t>(idx[r]) * row_words + w];
}

__global__ void gather_u32_kernel(const uint32_t* __restrict__ src, const uint32_t* __restrict__ idx, uint64_t rows,
                                  uint32_t* __restrict__ dst) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t < rows) dst[t] = src[idx[t]];
}

void gather_rows(const void* src, const uint32_t* idx, size_t rows, size_t row_bytes, void* dst,
                 cudaStream_t stream) {
    if (rows == 0 || row_bytes == 0) return;
    const uint64_t words = static_cast<uint64_t>(rows) * (row_bytes / 16);
    Profiler::Scope prof("compact_rows", stream, rows);
    gather_row_bytes_kernel<<<static_cast<uint32_t>((words + 255) / 256), 256, 0, stream>>>(
        static_cast<const uint4*>(src), idx, rows, static_cast<uint32_t>(row_bytes / 16), static_cast<uint4*>(dst));
    check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "compaction kernel");
}

constexpr uint32_t kBlobMagic = 0x58324245u;  // "EB2X"
constexpr uint32_t kBlobVersion = 1;

struct BlobHeader {
    uint32_t magic, version;
    int32_t metric, precision;
    uint32_t dim, d_pad, elem_bytes, flags;  // flags: 1 = lo plane, 2 = norms, 4 = removal bits
    uint64_t rows, removed;
};

}  // namespace

void ExactIndex::compact(uint32_t* new_to_old) {
    DeviceGuard g(device_);
    check_cuda(cudaDeviceSynchronize(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "compact sync");
    const size_t keep = live();
    std::vector<uint32_t> order;
    order.reserve(keep);
    for (size_t r = 0; r < n_; ++r)
        if (live_.get() == nullptr || ((live_host_[r >> 5] >> (r & 31)) & 1u)) order.push_back(static_cast<uint32_t>(r));
    if (new_to_old != nullptr) std::copy(order.begin(), order.end(), new_to_old);
    if (removed_ == 0) return;
    const size_t cap = std::max<size_t>(keep, 1);
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    DeviceBuffer idx(device_, cap * 4);
    DeviceBuffer ops(device_, cap * row_bytes);
    DeviceBuffer lo(device_, ops_lo_.get() ? cap * row_bytes : 0);
    DeviceBuffer norms(device_, norms_.get() ? cap * sizeof(float) : 0);
    if (keep > 0) {
        check_cuda(cudaMemcpy(idx.get(), order.data(), keep * 4, cudaMemcpyHostToDevice), ELIPS_B200_TRANSFER_FAILED,
                   "order upload");
        const uint32_t* ix = static_cast<const uint32_t*>(idx.get());
        gather_rows(ops_.get(), ix, keep, row_bytes, ops.get(), nullptr);
        if (lo.get()) gather_rows(ops_lo_.get(), ix, keep, row_bytes, lo.get(), nullptr);
        if (norms.get()) {
            gather_u32_kernel<<<static_cast<uint32_t>((keep + 255) / 256), 256>>>(
                static_cast<const uint32_t*>(norms_.get()), ix, keep, static_cast<uint32_t*>(norms.get()));
            check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "compaction kernel");
        }
        check_cuda(cudaDeviceSynchronize(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "compaction");
    }
    ops_ = std::move(ops);
    ops_lo_ = std::move(lo);
    norms_ = std::move(norms);
    capacity_ = cap;
    n_ = keep;
    removed_ = 0;
    live_ = DeviceBuffer();
    live_host_.clear();
}

size_t ExactIndex::device_bytes() const {
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    return capacity_ * row_bytes * (ops_lo_.get() ? 2 : 1) + (norms_.get() ? capacity_ * 4 : 0) +
           (live_.get() ? live_host_.size() * 4 : 0);
}

size_t ExactIndex::blob_bytes() const {
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    return sizeof(BlobHeader) + n_ * row_bytes * (ops_lo_.get() ? 2 : 1) + (norms_.get() ? n_ * 4 : 0) +
           (live_.get() ? live_host_.size() * 4 : 0);
}

void ExactIndex::export_blob(void* out, size_t bytes) const {
    if (out == nullptr || bytes < blob_bytes()) fail(ELIPS_B200_INVALID_ARGUMENT, "snapshot buffer too small");
    DeviceGuard g(device_);
    check_cuda(cudaDeviceSynchronize(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "export sync");
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    BlobHeader h{kBlobMagic, kBlobVersion, metric_, precision_, dim_, d_pad_, elem_bytes_,
                 (ops_lo_.get() ? 1u : 0u) | (norms_.get() ? 2u : 0u) | (live_.get() ? 4u : 0u), n_, removed_};
    uint8_t* o = static_cast<uint8_t*>(out);
    std::memcpy(o, &h, sizeof(h));
    o += sizeof(h);
    auto down = [&](const DeviceBuffer& b, size_t nbytes) {
        if (nbytes == 0) return;
        check_cuda(cudaMemcpy(o, b.get(), nbytes, cudaMemcpyDeviceToHost), ELIPS_B200_TRANSFER_FAILED, "snapshot");
        o += nbytes;
    };
    down(ops_, n_ * row_bytes);
    if (ops_lo_.get()) down(ops_lo_, n_ * row_bytes);
    if (norms_.get()) down(norms_, n_ * 4);
    if (live_.get()) {
        std::memcpy(o, live_host_.data(), live_host_.size() * 4);
        o += live_host_.size() * 4;
    }
}

void ExactIndex::import_blob(const void* blob, size_t bytes) {
    if (blob == nullptr || bytes < sizeof(BlobHeader)) fail(ELIPS_B200_INVALID_ARGUMENT, "snapshot too short");
    if (n_ != 0) fail(ELIPS_B200_INVALID_ARGUMENT, "snapshots load into an empty index");
    BlobHeader h;
    std::memcpy(&h, blob, sizeof(h));
    if (h.magic != kBlobMagic || h.version != kBlobVersion) fail(ELIPS_B200_INVALID_ARGUMENT, "not an index snapshot");
    if (h.metric != metric_ || h.precision != precision_ || h.dim != dim_ || h.d_pad != d_pad_ ||
        h.elem_bytes != elem_bytes_)
        fail(ELIPS_B200_DIMENSION_MISMATCH, "snapshot of a different metric, precision or dimension");
    const bool has_lo = (h.flags & 1u) != 0, has_norms = (h.flags & 2u) != 0, has_live = (h.flags & 4u) != 0;
    if (has_lo != (kind_ == OperandKind::TF32X3) || has_norms != (metric_ == kEuclidean))
        fail(ELIPS_B200_INVALID_ARGUMENT, "snapshot planes do not match the index");
    const size_t rows = h.rows, row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    const size_t words = (rows + 31) / 32;
    const size_t need = sizeof(h) + rows * row_bytes * (has_lo ? 2 : 1) + (has_norms ? rows * 4 : 0) +
                        (has_live ? words * 4 : 0);
    if (bytes < need) fail(ELIPS_B200_INVALID_ARGUMENT, "snapshot truncated");
    if (rows >= 0xFFFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "index limited to 2^32-2 rows");
    DeviceGuard g(device_);
    reserve(std::max<size_t>(rows, 1));
    const uint8_t* in = static_cast<const uint8_t*>(blob) + sizeof(h);
    auto up = [&](DeviceBuffer& b, size_t nbytes) {
        if (nbytes == 0) return;
        check_cuda(cudaMemcpy(b.get(), in, nbytes, cudaMemcpyHostToDevice), ELIPS_B200_TRANSFER_FAILED, "snapshot");
        in += nbytes;
    };
    up(ops_, rows * row_bytes);
    if (has_lo) up(ops_lo_, rows * row_bytes);
    if (has_norms) up(norms_, rows * 4);
    n_ = rows;
    if (has_live) {
        live_ = DeviceBuffer(device_, (capacity_ + 31) / 32 * 4);
        live_host_.assign(reinterpret_cast<const uint32_t*>(in), reinterpret_cast<const uint32_t*>(in) + words);
        removed_ = 0;
        for (size_t r = 0; r < rows; ++r) removed_ += ((live_host_[r >> 5] >> (r & 31)) & 1u) ? 0 : 1;
        if (removed_ != h.removed) fail(ELIPS_B200_INVALID_ARGUMENT, "snapshot removal bits inconsistent");
        upload_live_words(0, words);
    }
}

bool ExactIndex::remove(size_t row) {
    if (row >= n_) fail(ELIPS_B200_INVALID_ARGUMENT, "row out of range");
    DeviceGuard g(device_);
    // Searches still running on any stream may be reading the bits.
    check_cuda(cudaDeviceSynchronize(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "remove sync");
    if (live_.get() == nullptr) {
        live_ = DeviceBuffer(device_, (capacity_ + 31) / 32 * 4);
        live_host_.assign((n_ + 31) / 32, 0u);
        for (size_t r = 0; r < n_; ++r) live_host_[r >> 5] |= 1u << (r & 31);
        upload_live_words(0, live_host_.size());
    }
    uint32_t& w = live_host_[row >> 5];
    const uint32_t bit = 1u << (row & 31);
    if ((w & bit) == 0) return false;
    w &= ~bit;
    ++removed_;
    upload_live_words(row >> 5, (row >> 5) + 1);
    return true;
}

void ExactIndex::add(const void* rows_host, size_t n) {
    if (n == 0) return;
    if (rows_host == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "rows is null");
    if (n_ + n >= 0xFFFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "index limited to 2^32-2 rows");
    DeviceGuard g(device_);
    reserve(n_ + n);
    const size_t in_elem = kind_ == OperandKind::I8 ? 1 : 4;
    const size_t in_row = static_cast<size_t>(dim_) * in_elem;
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    // Stage through a bounded device buffer: 64 MiB of input rows at a time.
    const size_t chunk = std::max<size_t>(1, (64ull << 20) / in_row);
    cudaStream_t stream = nullptr;
    check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), ELIPS_B200_INITIALIZATION_FAILED,
               "cudaStreamCreate");
    try {
        DeviceBuffer staging(device_, std::min(chunk, n) * in_row);
        for (size_t r0 = 0; r0 < n; r0 += chunk) {
            const size_t rows = std::min(chunk, n - r0);
            check_cuda(cudaMemcpyAsync(staging.get(), static_cast<const uint8_t*>(rows_host) + r0 * in_row,
                                       rows * in_row, cudaMemcpyHostToDevice, stream),
                       ELIPS_B200_TRANSFER_FAILED, "row upload");
            const size_t dst = n_ + r0;
            prep_operands(kind_, staging.get(), rows, dim_, d_pad_,
                          static_cast<uint8_t*>(ops_.get()) + dst * row_bytes,
                          ops_lo_.get() ? static_cast<uint8_t*>(ops_lo_.get()) + dst * row_bytes : nullptr,
                          norms_.get() ? static_cast<float*>(norms_.get()) + dst : nullptr, stream);
            check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "row prep");
        }
    } catch (...) {
        cudaStreamDestroy(stream);
        throw;
    }
    cudaStreamDestroy(stream);
    mark_live(n_, n);
    n_ += n;
}

void ExactIndex::add_device(const void* rows, size_t n, cudaStream_t stream) {
    if (n == 0) return;
    if (rows == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "rows is null");
    if (n_ + n >= 0xFFFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "index limited to 2^32-2 rows");
    DeviceGuard g(device_);
    // Growing reallocates; finish work already queued on `stream` first.
    check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "add_device sync");
    reserve(n_ + n);
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    prep_operands(kind_, rows, n, dim_, d_pad_, static_cast<uint8_t*>(ops_.get()) + n_ * row_bytes,
                  ops_lo_.get() ? static_cast<uint8_t*>(ops_lo_.get()) + n_ * row_bytes : nullptr,
                  norms_.get() ? static_cast<float*>(norms_.get()) + n_ : nullptr, stream);
    check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "row prep");
    mark_live(n_, n);
    n_ += n;
}

void ExactIndex::search_device(const void* queries, size_t nq, size_t k, const uint32_t* mask,
                               uint32_t row_offset, float* out_dist, int64_t* out_rows,
                               uint2* out_cand, cudaStream_t stream, uint32_t* shared_bound) const {
    if (nq == 0 || k == 0) return;
    if (k > kMaxK) fail(ELIPS_B200_INVALID_ARGUMENT, "k above 1024 is not supported");
    if (nq > 0x7FFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "too many queries in one call");
    if (queries == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "queries is null");
    DeviceGuard g(device_);
    const DeviceProps& props = device_props(device_);
    if (n_ == 0) {
        // Nothing to search: every slot is empty.
        merge_candidates(device_, nullptr, static_cast<uint32_t>(nq), 0, static_cast<uint32_t>(k), 0, 0,
                         metric_, out_dist, out_rows, out_cand, stream);
        return;
    }
    if (mask != nullptr && n_ >= kGatherMinRows &&
        search_gathered(queries, nq, k, mask, row_offset, out_dist, out_rows, out_cand, stream, shared_bound))
        return;
    const RowView own{ops_.get(), ops_lo_.get(), static_cast<const float*>(norms_.get()),
                      static_cast<const uint32_t*>(live_.get()), static_cast<uint32_t>(n_)};
    search_rows(own, queries, nq, k, mask, row_offset, out_dist, out_rows, out_cand, stream, shared_bound);
}

bool ExactIndex::search_gathered(const void* queries, size_t nq, size_t k, const uint32_t* mask,
                                 uint32_t row_offset, float* out_dist, int64_t* out_rows, uint2* out_cand,
                                 cudaStream_t stream, uint32_t* shared_bound) const {
    const uint32_t n = static_cast<uint32_t>(n_);
    const uint32_t nwords = (n + 31u) / 32u;
    const uint32_t* live = static_cast<const uint32_t*>(live_.get());
    auto align = [](size_t x) { return (x + 255) / 256 * 256; };
    // The selected rows (at most n / 2 are kept; more and the whole base is
    // searched) and their count, read back to size the subset and its plan.
    const uint32_t cap = n / 2u + 1u;
    const uint32_t blocks = (nwords + kSelectThreads - 1) / kSelectThreads;
    const size_t rows_b = align(static_cast<size_t>(cap) * sizeof(uint32_t));
    StreamScratch sel(rows_b + align(static_cast<size_t>(blocks) * sizeof(uint32_t)) + 256, stream);
    uint32_t* rows = reinterpret_cast<uint32_t*>(sel.get());
    uint32_t* block_counts = reinterpret_cast<uint32_t*>(sel.get() + rows_b);
    uint32_t* total = block_counts + align(static_cast<size_t>(blocks) * sizeof(uint32_t)) / sizeof(uint32_t);
    {
        Profiler::Scope prof("mask_select", stream, nwords);
        select_count_kernel<<<blocks, kSelectThreads, 0, stream>>>(mask, live, n, nwords, block_counts);
        select_rows_kernel<<<blocks, kSelectThreads, 0, stream>>>(mask, live, n, nwords, block_counts, rows, cap,
                                                                  total);
        check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "row selection launch");
    }
    uint32_t m = 0;
    check_cuda(cudaMemcpyAsync(&m, total, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream),
               ELIPS_B200_TRANSFER_FAILED, "selected count");
    check_cuda(cudaStreamSynchronize(stream), ELIPS_B200_KERNEL_LAUNCH_FAILED, "selected count");
    if (static_cast<uint64_t>(m) * 2 > n) return false;
    if (m == 0) {
        merge_candidates(device_, nullptr, static_cast<uint32_t>(nq), 0, static_cast<uint32_t>(k), 0, 0, metric_,
                         out_dist, out_rows, out_cand, stream);
        return true;
    }
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    const size_t ops_b = align(static_cast<size_t>(m) * row_bytes);
    const size_t lo_b = ops_lo_.get() ? ops_b : 0;
    const size_t norms_b = norms_.get() ? align(static_cast<size_t>(m) * sizeof(float)) : 0;
    StreamScratch sub(ops_b + lo_b + norms_b, stream);
    uint8_t* g_ops = sub.get();
    uint8_t* g_lo = lo_b ? g_ops + ops_b : nullptr;
    float* g_norms = norms_b ? reinterpret_cast<float*>(g_ops + ops_b + lo_b) : nullptr;
    {
        Profiler::Scope prof("mask_gather", stream, static_cast<uint64_t>(m) * row_bytes);
        const uint64_t warps = (static_cast<uint64_t>(m) + kGatherRowsPerWarp - 1) / kGatherRowsPerWarp;
        const uint32_t blocks = static_cast<uint32_t>((warps * 32 + 255) / 256);
        gather_rows_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(ops_.get()), g_ops, rows, m,
                                                       static_cast<uint32_t>(row_bytes),
                                                       static_cast<const float*>(norms_.get()), g_norms);
        if (g_lo != nullptr)
            gather_rows_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(ops_lo_.get()), g_lo, rows,
                                                           m, static_cast<uint32_t>(row_bytes), nullptr, nullptr);
        check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "gather launch");
    }
    const RowView subset{g_ops, g_lo, g_norms, nullptr, m};
    search_rows(subset, queries, nq, k, nullptr, 0, out_dist, out_rows, out_cand, stream, shared_bound);
    const size_t count = nq * k;
    remap_rows_kernel<<<static_cast<uint32_t>((count + 255) / 256), 256, 0, stream>>>(out_rows, out_cand, count,
                                                                                       rows, row_offset);
    check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "remap launch");
    return true;
}

void ExactIndex::search_rows(const RowView& rv, const void* queries, size_t nq, size_t k, const uint32_t* mask,
                             uint32_t row_offset, float* out_dist, int64_t* out_rows, uint2* out_cand,
                             cudaStream_t stream, uint32_t* shared_bound) const {
    const DeviceProps& props = device_props(device_);
    const uint32_t n = rv.n;
    // More than one 128-query tile: CTA pairs (M = 256 per MMA).
    const bool pair = nq > kTileM;
    const ExactPlan plan = plan_exact(static_cast<uint32_t>(nq), n, static_cast<uint32_t>(k), bn_of(kind_),
                                      pair ? pair_groups(device_) : props.num_sms, pair ? 2u : 1u);
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    auto align = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t q_ops = align(nq * row_bytes);
    const size_t q_lo = kind_ == OperandKind::TF32X3 ? q_ops : 0;
    const size_t q_norm = metric_ == kEuclidean ? align(nq * sizeof(float)) : 0;
    const size_t cand = align(static_cast<size_t>(plan.grid) * 2 * kTileM * plan.cap * sizeof(uint2));
    const uint32_t slot = publish_slot(plan, static_cast<uint32_t>(nq), static_cast<uint32_t>(k));
    const size_t partial = align(nq * plan.splits * 2 * slot * sizeof(uint2));
    const size_t qtau = align(nq * sizeof(uint32_t));
    const uint32_t n_lists = plan.splits * 2;
    const uint32_t merge_group = merge_group_size(static_cast<uint32_t>(nq), n_lists, slot, props.num_sms);
    const uint32_t groups = merge_group < n_lists ? (n_lists + merge_group - 1) / merge_group : 0;
    const size_t stage = align(static_cast<size_t>(nq) * groups * k * sizeof(uint2));
    StreamScratch scratch(q_ops + q_lo + q_norm + cand + partial + qtau + stage, stream);
    uint8_t* s = scratch.get();
    void* qa = s;
    void* qlo = q_lo ? s + q_ops : nullptr;
    float* qn = q_norm ? reinterpret_cast<float*>(s + q_ops + q_lo) : nullptr;
    uint2* cand_buf = reinterpret_cast<uint2*>(s + q_ops + q_lo + q_norm);
    uint2* part_buf = reinterpret_cast<uint2*>(s + q_ops + q_lo + q_norm + cand);
    uint32_t* qtau_buf = reinterpret_cast<uint32_t*>(s + q_ops + q_lo + q_norm + cand + partial);
    if (shared_bound != nullptr) qtau_buf = shared_bound;
    else
        check_cuda(cudaMemsetAsync(qtau_buf, 0xFF, nq * sizeof(uint32_t), stream), ELIPS_B200_KERNEL_LAUNCH_FAILED,
                   "threshold init");
    prep_operands(kind_, queries, nq, dim_, d_pad_, qa, qlo, qn, stream);

    const CUtensorMapDataType dt = tma_dtype_of(kind_);
    const CUtensorMap ma = make_operand_map(qa, dt, elem_bytes_, d_pad_, nq, kTileM);
    const CUtensorMap mb = make_operand_map(rv.ops, dt, elem_bytes_, d_pad_, n, plan.bn / plan.cg);
    CUtensorMap malo = ma, mblo = mb;
    if (kind_ == OperandKind::TF32X3) {
        malo = make_operand_map(qlo, dt, elem_bytes_, d_pad_, nq, kTileM);
        mblo = make_operand_map(rv.ops_lo, dt, elem_bytes_, d_pad_, n, plan.bn / plan.cg);
    }
    ExactParams prm{};
    prm.base_norms = rv.norms;
    prm.query_norms = qn;
    prm.mask = mask;
    prm.live = rv.live;
    prm.cand = cand_buf;
    prm.partial = part_buf;
    prm.qtau = qtau_buf;
    prm.n = n;
    prm.nq = static_cast<uint32_t>(nq);
    prm.k = static_cast<uint32_t>(k);
    prm.cap = plan.cap;
    prm.splits = plan.splits;
    prm.n_qt = plan.n_qt;
    prm.n_bt = plan.n_bt;
    prm.num_units = plan.n_qt * plan.splits;
    prm.kblocks = d_pad_ * elem_bytes_ / kKBlockBytes;
    prm.slot = slot;
    prm.early = early_compaction(static_cast<uint32_t>(k), plan);
    prm.row_offset = row_offset;
    prm.metric = metric_;
    dispatch_exact(kind_, metric_, ma, mb, malo, mblo, prm, plan, stream);
    uint2* stage_buf = reinterpret_cast<uint2*>(s + q_ops + q_lo + q_norm + cand + partial + qtau);
    merge_split_lists(device_, part_buf, stage_buf, static_cast<uint32_t>(nq), n_lists, merge_group, groups,
                      static_cast<uint32_t>(k), metric_, out_dist, out_rows, out_cand, stream, slot);
}

void ExactIndex::search_device_in_scratch(const void* queries, size_t nq, size_t k, const uint32_t* mask,
                                          float* out_dist, int64_t* out_rows, uint8_t* scratch,
                                          size_t scratch_bytes, uint32_t max_grid,
                                          cudaStream_t stream) const {
    if (nq == 0 || k == 0) return;
    if (k > kMaxK) fail(ELIPS_B200_INVALID_ARGUMENT, "k above 1024 is not supported");
    if (nq > 0x7FFFFFFFull) fail(ELIPS_B200_INVALID_ARGUMENT, "too many queries in one call");
    if (queries == nullptr) fail(ELIPS_B200_INVALID_ARGUMENT, "queries is null");
    if (scratch == nullptr || max_grid == 0) fail(ELIPS_B200_INVALID_ARGUMENT, "no scratch buffer");
    DeviceGuard g(device_);
    const DeviceProps& props = device_props(device_);
    if (n_ == 0) {
        merge_candidates(device_, nullptr, static_cast<uint32_t>(nq), 0, static_cast<uint32_t>(k), 0, 0,
                         metric_, out_dist, out_rows, nullptr, stream);
        return;
    }
    const uint32_t n = static_cast<uint32_t>(n_);
    const int ctas = static_cast<int>(std::min<uint32_t>(max_grid, static_cast<uint32_t>(props.num_sms)));
    const ExactPlan plan = plan_exact(static_cast<uint32_t>(nq), n, static_cast<uint32_t>(k), bn_of(kind_), ctas);
    const size_t row_bytes = static_cast<size_t>(d_pad_) * elem_bytes_;
    auto align = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t q_ops = align(nq * row_bytes);
    const size_t q_lo = kind_ == OperandKind::TF32X3 ? q_ops : 0;
    const size_t q_norm = metric_ == kEuclidean ? align(nq * sizeof(float)) : 0;
    const size_t cand = align(static_cast<size_t>(plan.grid) * 2 * kTileM * plan.cap * sizeof(uint2));
    const size_t partial = align(nq * plan.splits * 2 * k * sizeof(uint2));
    const size_t qtau = align(nq * sizeof(uint32_t));
    const uint32_t n_lists = plan.splits * 2;
    const uint32_t merge_group = merge_group_size(static_cast<uint32_t>(nq), n_lists, static_cast<uint32_t>(k),
                                                  props.num_sms);
    const uint32_t groups = merge_group < n_lists ? (n_lists + merge_group - 1) / merge_group : 0;
    const size_t stage = align(static_cast<size_t>(nq) * groups * k * sizeof(uint2));
    const size_t need = q_ops + q_lo + q_norm + cand + partial + qtau + stage;
    if (need > scratch_bytes)
        fail(ELIPS_B200_INVALID_ARGUMENT,
             "search needs " + std::to_string(need >> 20) + " MiB of scratch, above the " +
                 std::to_string(scratch_bytes >> 20) + " MiB fixed buffer; split the query batch");
    uint8_t* s = scratch;
    void* qa = s;
    void* qlo = q_lo ? s + q_ops : nullptr;
    float* qn = q_norm ? reinterpret_cast<float*>(s + q_ops + q_lo) : nullptr;
    uint2* cand_buf = reinterpret_cast<uint2*>(s + q_ops + q_lo + q_norm);
    uint2* part_buf = reinterpret_cast<uint2*>(s + q_ops + q_lo + q_norm + cand);
    uint32_t* qtau_buf = reinterpret_cast<uint32_t*>(s + q_ops + q_lo + q_norm + cand + partial);
    // The buffer keeps the previous call's contents: the shared bounds must
    // start at "no bound"; the lists and partial outputs are always written
    // before they are read.
    check_cuda(cudaMemsetAsync(qtau_buf, 0xFF, nq * sizeof(uint32_t), stream), ELIPS_B200_KERNEL_LAUNCH_FAILED,
               "threshold init");
    prep_operands(kind_, queries, nq, dim_, d_pad_, qa, qlo, qn, stream);
    const CUtensorMapDataType dt = tma_dtype_of(kind_);
    const CUtensorMap ma = make_operand_map(qa, dt, elem_bytes_, d_pad_, nq, kTileM);
    const CUtensorMap mb = make_operand_map(ops_.get(), dt, elem_bytes_, d_pad_, n, plan.bn / plan.cg);
    CUtensorMap malo = ma, mblo = mb;
    if (kind_ == OperandKind::TF32X3) {
        malo = make_operand_map(qlo, dt, elem_bytes_, d_pad_, nq, kTileM);
        mblo = make_operand_map(ops_lo_.get(), dt, elem_bytes_, d_pad_, n, plan.bn / plan.cg);
    }
    ExactParams prm{};
    prm.base_norms = static_cast<const float*>(norms_.get());
    prm.query_norms = qn;
    prm.mask = mask;
    prm.live = static_cast<const uint32_t*>(live_.get());
    prm.cand = cand_buf;
    prm.partial = part_buf;
    prm.qtau = qtau_buf;
    prm.n = n;
    prm.nq = static_cast<uint32_t>(nq);
    prm.k = static_cast<uint32_t>(k);
    prm.cap = plan.cap;
    prm.splits = plan.splits;
    prm.n_qt = plan.n_qt;
    prm.n_bt = plan.n_bt;
    prm.num_units = plan.n_qt * plan.splits;
    prm.kblocks = d_pad_ * elem_bytes_ / kKBlockBytes;
    prm.row_offset = 0;
    prm.slot = prm.k;
    prm.metric = metric_;
    dispatch_exact(kind_, metric_, ma, mb, malo, mblo, prm, plan, stream);
    uint2* stage_buf = reinterpret_cast<uint2*>(s + q_ops + q_lo + q_norm + cand + partial + qtau);
    merge_split_lists(device_, part_buf, stage_buf, static_cast<uint32_t>(nq), n_lists, merge_group, groups,
                      static_cast<uint32_t>(k), metric_, out_dist, out_rows, nullptr, stream,
                      static_cast<uint32_t>(k));
}

void merge_candidates(int device, const uint2* cand, uint32_t nq, uint32_t lists, uint32_t k,
                      uint64_t stride_q, uint64_t stride_l, int metric, float* out_dist,
                      int64_t* out_rows, uint2* out_cand, cudaStream_t stream, uint32_t sub,
                      uint32_t lists_last, uint32_t len) {
    if (len == 0) len = k;
    if (nq == 0 || k == 0) return;
    if (sub == 0) sub = 1;
    if (sub == 1 || lists_last == 0) lists_last = lists;
    if (k > kMaxK) fail(ELIPS_B200_INVALID_ARGUMENT, "k above 1024 is not supported");
    uint32_t kpow2 = 1;
    while (kpow2 < k) kpow2 <<= 1;
    constexpr uint32_t warps = 4;
    // Up to 2048 candidates per query (16 KB) stay in shared memory for all
    // selection passes; larger merges read global memory on every pass.
    const uint64_t count = static_cast<uint64_t>(std::max(lists, lists_last)) * len;
    const uint32_t cache_cap = count <= kMergeCacheMax ? static_cast<uint32_t>((count + 1) / 2 * 2) : 0u;
    const size_t smem = warps * (1024 + static_cast<size_t>(kpow2) * 8 + static_cast<size_t>(cache_cap) * 8);
    allow_dynamic_smem(reinterpret_cast<const void*>(merge_topk_kernel), smem);
    const uint64_t rows_out = static_cast<uint64_t>(nq) * sub;
    const uint32_t blocks = static_cast<uint32_t>((rows_out + warps - 1) / warps);
    Profiler::Scope prof("merge_topk", stream, static_cast<uint64_t>(nq) * ((sub - 1) * lists + lists_last) * len);
    merge_topk_kernel<<<blocks, warps * 32, smem, stream>>>(cand, nq, lists, k, len, stride_q, stride_l, kpow2,
                                                           cache_cap, sub, lists_last, metric, out_dist,
                                                           out_rows, out_cand);
    check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "merge kernel launch");
}

namespace {

// One thread waits on an mbarrier that nothing arrives on, for `budget`
// cycles: the bounded wait expires, records the device error word and raises
// the CTA's abort flag, the path every pipeline wait takes when a producer or
// consumer is lost. Nothing asynchronous is in flight, so returning with the
// barrier pending is safe.
__global__ void wait_selftest_kernel(long long budget) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x != 0) return;
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbarrier_init();
    mbar_wait_for(smem_u32(&bar), 0, &abort_flag, budget);
}

}  // namespace

int wait_selftest(int device, long long budget) {
    if (budget < 1 || budget > kWaitTimeoutCycles)
        fail(ELIPS_B200_INVALID_ARGUMENT, "wait budget must be in [1, 2^31] cycles");
    DeviceGuard g(device);
    // start from a clear error word so the result is this launch's
    read_and_clear_device_error(device);
    wait_selftest_kernel<<<1, 32>>>(budget);
    check_cuda(cudaGetLastError(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "wait self-test launch");
    return read_and_clear_device_error(device);
}

int read_and_clear_device_error(int device) {
    DeviceGuard g(device);
    check_cuda(cudaDeviceSynchronize(), ELIPS_B200_KERNEL_LAUNCH_FAILED, "cudaDeviceSynchronize");
    int code = 0;
    check_cuda(cudaMemcpyFromSymbol(&code, g_device_error, sizeof(int)), ELIPS_B200_TRANSFER_FAILED,
               "read device error");
    const int zero = 0;
    check_cuda(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)), ELIPS_B200_TRANSFER_FAILED,
               "clear device error");
    return code;
}

}  // namespace eb
