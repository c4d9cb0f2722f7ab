// Fused exact k-NN search: query-tile x base-tile distance GEMM on the
// tcgen05 tensor cores with the accumulator in TMEM, and a per-query top-k
// filter fused into the TMEM read-back, so the Q x N distance matrix never
// reaches HBM.
//
// Replaces the reference's exhaustive scan ExactIndex::search
// (src/ExactIndex.cpp:55-87) and the GpuPort::compute_distances_batch +
// top_k pair that GpuBruteForceIndex::search_batch chains through a host
// Q x N matrix (src/gpu_engine/GpuSearchPipeline.cpp:10-41).
//
// Work decomposition. Queries are tiled by 128 (one TMEM lane each), base rows
// by BN. The base is cut into S contiguous splits; a work unit is one
// (query tile, split) pair and writes that split's candidates per query and
// column half to `partial[q][s][h][0..slot)`: its k best, or, when a list
// holds at most `slot` >= k entries, all of them, padded. Units are ordered
// split-major so the CTAs
// resident at any time share the same base region, which then streams from
// HBM once and is re-read from L2 by every query tile.
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM allocator and
// MMA issuer, warps 2-9 = epilogue. Two epilogue warps share each 32-lane
// TMEM quadrant and split the tile's columns in halves; a thread owns one
// (query, column half) pair and its own candidate list.
//
// CTA pairs (CG = 2). Two CTAs of a cluster run one M = 256 MMA per step
// (tcgen05 cta_group::2): each CTA loads its own 128 queries and its own half
// of the BN base rows, rank 0 issues the MMAs over both CTAs' shared memory
// and each CTA's TMEM receives its 128 queries x BN distances. Per CTA, a
// pipeline stage then carries A + B/2 instead of A + B, which is what bounds
// the single-CTA kernel (operand traffic from L2). Rank 0's barriers gate the
// MMA: the peer's loads complete on rank 0's full barrier, the MMA commit
// releases the stage in both CTAs, and the peer's epilogue warps release the
// accumulator on rank 0's barrier.
#pragma once

#include <cstdint>

#include "ptx.cuh"
#include "select.cuh"

namespace eb {

enum class OperandKind : int { F16 = 0, BF16 = 1, TF32X3 = 2, I8 = 3 };

enum MetricId : int { kCosine = 0, kEuclidean = 1, kDot = 2 };  // elips::Metric order

constexpr int kTileM = 128;           // queries per tile = TMEM lanes
constexpr int kKBlockBytes = 128;     // K bytes per pipeline stage (one swizzle atom)
constexpr int kEpilogueWarps = 8;
// Admission staging: a lane's 16 accumulator words of one half-chunk, padded
// to 20 words so the 16-byte stores of 8 consecutive lanes hit distinct banks.
constexpr uint32_t kStageStride = 20;
constexpr int kExactThreads = 32 * (2 + kEpilogueWarps);

struct ExactParams {
    const float* base_norms;   // [n] squared norms (euclidean only)
    const float* query_norms;  // [nq] squared norms (euclidean only)
    const uint32_t* mask;      // [ceil(n/32)] eligibility bits, or null
    const uint32_t* live;      // [ceil(n/32)] 0 bits = removed rows, or null (none removed)
    uint2* cand;               // [gridDim.x][2][128][cap] candidate lists per (column half, query)
    uint2* partial;            // [nq][splits][2][slot]
    uint32_t* qtau;            // [nq] shared admission bound per query (ordered key)
    uint32_t n, nq, k, cap, splits, n_qt, n_bt, num_units, kblocks;
    uint32_t slot;             // entries per published list, k <= slot <= cap
    uint32_t early;            // first compaction of a list in a unit once it holds more (0: none early)
    uint32_t row_offset;       // added to every emitted row (shard base)
    int metric;
};

template <OperandKind KIND>
struct KindTraits;
template <>
struct KindTraits<OperandKind::F16> {
    static constexpr MmaKind mma = MmaKind::F16;
    static constexpr uint32_t idesc_fmt = 0, c_fmt = 1, elem_bytes = 2;
    static constexpr bool x3 = false, integer = false;
};
template <>
struct KindTraits<OperandKind::BF16> {
    static constexpr MmaKind mma = MmaKind::F16;
    static constexpr uint32_t idesc_fmt = 1, c_fmt = 1, elem_bytes = 2;
    static constexpr bool x3 = false, integer = false;
};
template <>
struct KindTraits<OperandKind::TF32X3> {
    static constexpr MmaKind mma = MmaKind::TF32;
    static constexpr uint32_t idesc_fmt = 2, c_fmt = 1, elem_bytes = 4;
    static constexpr bool x3 = true, integer = false;
};
template <>
struct KindTraits<OperandKind::I8> {
    static constexpr MmaKind mma = MmaKind::I8;
    static constexpr uint32_t idesc_fmt = 1, c_fmt = 2, elem_bytes = 1;
    static constexpr bool x3 = false, integer = true;
};

template <OperandKind KIND, int BN, int STAGES, int CG = 1>
struct ExactConfig {
    using T = KindTraits<KIND>;
    static constexpr uint32_t kBRows = BN / CG;  // base rows this CTA loads per tile
    static constexpr uint32_t kABytes = kTileM * kKBlockBytes;
    static constexpr uint32_t kBBytes = kBRows * kKBlockBytes;
    static constexpr uint32_t kOperands = T::x3 ? 2 : 1;
    static constexpr uint32_t kStageBytes = (kABytes + kBBytes) * kOperands;
    static constexpr uint32_t kTmemCols = 2 * BN;
    static constexpr uint32_t kElemsPerKBlock = kKBlockBytes / T::elem_bytes;
    // barriers: full[S], empty[S], tfull[2], tempty[2], mma_done
    static constexpr uint32_t kBarBytes = 8 * (2 * STAGES + 5);
    static constexpr uint32_t kMiscOffset = STAGES * kStageBytes;
    // Per epilogue warp: the compaction histogram (256 words) and, never at
    // the same time, the admission staging rows (32 lanes x kStageStride words).
    static constexpr uint32_t kWarpScratchBytes = 32u * kStageStride * 4u > 1024u ? 32u * kStageStride * 4u : 1024u;
    static constexpr uint32_t kHistOffset = kMiscOffset + 256;
    static constexpr uint32_t kNormOffset = kHistOffset + kEpilogueWarps * kWarpScratchBytes;  // per-warp norms
    static constexpr uint32_t kSmemBytes = 1024 /* alignment slack */ + kNormOffset + kEpilogueWarps * (BN / 2) * 4;
    static_assert(kBarBytes + 16 <= 256, "barrier area");
    static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");
};

__device__ __forceinline__ bool drain_wait(uint32_t bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > kWaitTimeoutCycles) {
            record_device_error(kDevErrWaitTimeout);
            return false;
        }
    }
    return true;
}

// Largest candidate list the register-resident compaction handles (16
// entries per lane); longer lists take the global-memory path.
constexpr uint32_t kRegListCap = 512;

// Reduces one query's list to its k best entries (whole warp).
__device__ __forceinline__ float compact_one(uint2* list, uint32_t count, uint32_t k, uint32_t cap,
                                             uint32_t* hist) {
    if (cap <= kRegListCap) return warp_compact_regs<kRegListCap / 32>(list, count, k, hist);
    return warp_compact_list(list, count, k, hist);
}

// Effective strict admission threshold: below this unit's own k-th key, and
// at or below the best k-th key any unit has published for the query (a
// candidate equal to another unit's bound may still precede that unit's
// entries in (key, row) order, so the shared bound admits equality).
__device__ __forceinline__ float admission_threshold(float tau_local, uint32_t shared_bound) {
    const uint32_t inf_key = 0xFF800000u;  // ordered_key(+inf)
    uint32_t t = ordered_key(tau_local);
    const uint32_t g = shared_bound == 0xFFFFFFFFu ? 0xFFFFFFFFu : shared_bound + 1u;
    t = min(t, g);
    t = min(t, inf_key);
    return key_to_float(t);
}

// Ordering key of one accumulator word: the distance before the final
// square root (euclidean), i.e. 1 - dot (cosine), -dot (dot product),
// (|x|^2 - 2 q.x) + |q|^2 (euclidean), -(int32 dot) for the int8 codec.
template <OperandKind KIND, int METRIC>
__device__ __forceinline__ float key_of(uint32_t v, float xn, float qn) {
    if constexpr (KindTraits<KIND>::integer) {
        return -static_cast<float>(static_cast<int32_t>(v));
    } else if constexpr (METRIC == kCosine) {
        return 1.0f - __uint_as_float(v);
    } else if constexpr (METRIC == kDot) {
        return -__uint_as_float(v);
    } else {
        return fmaf(-2.0f, __uint_as_float(v), xn) + qn;
    }
}

// Admission test in the accumulator domain, one compare per column. Every
// column whose key is below `thr` passes (the converse need not hold: the
// exact key is tested again before an append):
//  * cosine: fl(1 - v) < thr implies v > 1 - thr (real), so v > c with c one
//    ulp below fl(1 - thr);
//  * dot: -v < thr  <=>  v > -thr (negation is exact);
//  * int8: -(float)iv < thr  <=>  iv > floor(-thr) (|iv| < 2^24 converts exactly);
//  * euclidean: fl(fma(-2, v, xn) + qn) < thr implies fma(-2, v, xn) < thr - qn
//    (real), so compare with fl(thr - qn) rounded one ulp up.
template <OperandKind KIND, int METRIC>
struct Admission {
    float c;     // float cutoff (cosine / dot: v > c; euclidean: fma(-2, v, xn) < c)
    int32_t ic;  // int8: iv > ic
    __device__ __forceinline__ Admission(float thr, float qn) {
        if constexpr (KindTraits<KIND>::integer) {
            const float t = -thr;
            ic = t < -2147483520.0f ? INT32_MIN : (t >= 2147483520.0f ? INT32_MAX : static_cast<int32_t>(floorf(t)));
            c = 0.0f;
        } else if constexpr (METRIC == kCosine) {
            c = nextafterf(1.0f - thr, -__int_as_float(0x7f800000));
            ic = 0;
        } else if constexpr (METRIC == kDot) {
            c = -thr;
            ic = 0;
        } else {
            c = nextafterf(thr - qn, __int_as_float(0x7f800000));
            ic = 0;
        }
    }
    __device__ __forceinline__ bool pass(uint32_t v, float xn) const {
        if constexpr (KindTraits<KIND>::integer) return static_cast<int32_t>(v) > ic;
        else if constexpr (METRIC == kEuclidean) return fmaf(-2.0f, __uint_as_float(v), xn) < c;
        else return __uint_as_float(v) > c;
    }
};

template <OperandKind KIND, int BN, int STAGES, int METRIC, int CG = 1>
__global__ void __launch_bounds__(kExactThreads, 1)
    exact_topk_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_a_lo,
                      const __grid_constant__ CUtensorMap tm_b_lo, const __grid_constant__ ExactParams p) {
    using Cfg = ExactConfig<KIND, BN, STAGES, CG>;
    static_assert(CG == 1 || CG == 2, "one CTA or a CTA pair");
    using Tr = KindTraits<KIND>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (sbase - raw);

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    // Work is distributed over MMA groups: single CTAs, or CTA pairs.
    uint32_t rank = 0, group = blockIdx.x, groups = gridDim.x;
    if constexpr (CG == 2) {
        rank = cluster_ctarank();
        group = cluster_id_x();
        groups = cluster_count_x();
    }
    const bool leader = rank == 0;
    constexpr uint32_t kGroupM = kTileM * CG;  // queries per unit

    const uint32_t bar0 = sbase + Cfg::kMiscOffset;
    auto full_bar = [&](uint32_t s) { return bar0 + 8u * s; };
    auto empty_bar = [&](uint32_t s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](uint32_t a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](uint32_t a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
    const uint32_t mma_done_bar = bar0 + 8u * (2 * STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOffset + Cfg::kBarBytes);
    volatile int* abort_flag =
        reinterpret_cast<volatile int*>(smem + Cfg::kMiscOffset + Cfg::kBarBytes + 8);

    // stage s: A at s*stage, B after A (then A_lo, B_lo for the 3xTF32 split)
    auto a_addr = [&](uint32_t s) { return sbase + s * Cfg::kStageBytes; };
    auto b_addr = [&](uint32_t s) { return a_addr(s) + Cfg::kABytes; };
    auto alo_addr = [&](uint32_t s) { return b_addr(s) + Cfg::kBBytes; };
    auto blo_addr = [&](uint32_t s) { return alo_addr(s) + Cfg::kABytes; };

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (uint32_t a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), kEpilogueWarps * CG);
        }
        mbar_init(mma_done_bar, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        if constexpr (CG == 2) {
            tmem_alloc_pair(smem_u32(tmem_slot), Cfg::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    // The peer's barriers must be initialised before either CTA signals them.
    if constexpr (CG == 2) cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const uint32_t num_units = p.num_units;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one_sync()) {
            tma_prefetch_desc(&tm_a);
            tma_prefetch_desc(&tm_b);
            if constexpr (Tr::x3) {
                tma_prefetch_desc(&tm_a_lo);
                tma_prefetch_desc(&tm_b_lo);
            }
            uint32_t stage = 0, phase = 0;
            uint32_t issued_mask = 0, issued_parity = 0;
            bool ok = true;
            for (uint32_t unit = group; ok && unit < num_units; unit += groups) {
                const uint32_t qt = unit % p.n_qt, sp = unit / p.n_qt;
                const uint32_t bt0 = static_cast<uint32_t>((uint64_t)sp * p.n_bt / p.splits);
                const uint32_t bt1 = static_cast<uint32_t>((uint64_t)(sp + 1) * p.n_bt / p.splits);
                const int32_t a_row = static_cast<int32_t>(qt * kGroupM + rank * kTileM);
                for (uint32_t bt = bt0; ok && bt < bt1; ++bt) {
                    const int32_t b_row = static_cast<int32_t>(bt * BN + rank * Cfg::kBRows);
                    for (uint32_t kb = 0; kb < p.kblocks; ++kb) {
                        if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
                            ok = false;
                            break;
                        }
                        const int32_t x = static_cast<int32_t>(kb * Cfg::kElemsPerKBlock);
                        if constexpr (CG == 2) {
                            // Both halves complete on rank 0's barrier, which
                            // rank 0 arms with the bytes of both.
                            if (leader) mbar_arrive_expect_tx(full_bar(stage), 2u * Cfg::kStageBytes);
                            const uint32_t fb = mapa_shared(full_bar(stage), 0);
                            tma_load_2d_pair(a_addr(stage), &tm_a, fb, x, a_row);
                            tma_load_2d_pair(b_addr(stage), &tm_b, fb, x, b_row);
                            if constexpr (Tr::x3) {
                                tma_load_2d_pair(alo_addr(stage), &tm_a_lo, fb, x, a_row);
                                tma_load_2d_pair(blo_addr(stage), &tm_b_lo, fb, x, b_row);
                            }
                        } else {
                            mbar_arrive_expect_tx(full_bar(stage), Cfg::kStageBytes);
                            tma_load_2d(a_addr(stage), &tm_a, full_bar(stage), x, a_row);
                            tma_load_2d(b_addr(stage), &tm_b, full_bar(stage), x, b_row);
                            if constexpr (Tr::x3) {
                                tma_load_2d(alo_addr(stage), &tm_a_lo, full_bar(stage), x, a_row);
                                tma_load_2d(blo_addr(stage), &tm_b_lo, full_bar(stage), x, b_row);
                            }
                        }
                        issued_mask |= 1u << stage;
                        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            // Every load this thread issued must land before the CTA exits.
            // In a pair, rank 0's full barriers count the peer's bytes too,
            // and the peer leaves only after the closing cluster barrier.
            if (leader) {
                for (uint32_t s = 0; s < STAGES; ++s) {
                    if (issued_mask & (1u << s)) drain_wait(full_bar(s), (issued_parity >> s) & 1u);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (rank 0 of a pair)
        if (leader && elect_one_sync()) {
            constexpr uint32_t idesc = make_idesc(Tr::c_fmt, Tr::idesc_fmt, kGroupM, BN);
            uint32_t stage = 0, phase = 0, tile_iter = 0;
            bool ok = true;
            for (uint32_t unit = group; ok && unit < num_units; unit += groups) {
                const uint32_t sp = unit / p.n_qt;
                const uint32_t bt0 = static_cast<uint32_t>((uint64_t)sp * p.n_bt / p.splits);
                const uint32_t bt1 = static_cast<uint32_t>((uint64_t)(sp + 1) * p.n_bt / p.splits);
                for (uint32_t bt = bt0; ok && bt < bt1; ++bt, ++tile_iter) {
                    const uint32_t acc = tile_iter & 1u;
                    const uint32_t acc_phase = (tile_iter >> 1) & 1u;
                    const bool freed = CG == 2 ? mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1u, abort_flag)
                                               : mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag);
                    if (!freed) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * BN;
                    for (uint32_t kb = 0; kb < p.kblocks; ++kb) {
                        if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
#pragma unroll
                        for (uint32_t k = 0; k < 4; ++k) {
                            const uint32_t first = (kb == 0 && k == 0) ? 0u : 1u;
                            const uint64_t ad = smem_desc_k128(a_addr(stage) + 32u * k);
                            const uint64_t bd = smem_desc_k128(b_addr(stage) + 32u * k);
                            if constexpr (Tr::x3) {
                                const uint64_t adl = smem_desc_k128(alo_addr(stage) + 32u * k);
                                const uint64_t bdl = smem_desc_k128(blo_addr(stage) + 32u * k);
                                tc_mma<Tr::mma, CG>(d_tmem, adl, bd, idesc, first);
                                tc_mma<Tr::mma, CG>(d_tmem, ad, bdl, idesc, 1u);
                                tc_mma<Tr::mma, CG>(d_tmem, ad, bd, idesc, 1u);
                            } else {
                                tc_mma<Tr::mma, CG>(d_tmem, ad, bd, idesc, first);
                            }
                        }
                        if constexpr (CG == 2) tc_commit_pair_both(empty_bar(stage), 0x3);
                        else tc_commit(empty_bar(stage));
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    if constexpr (CG == 2) tc_commit_pair_both(tfull_bar(acc), 0x3);
                    else tc_commit(tfull_bar(acc));
                }
            }
            // All MMAs this thread issued must finish before TMEM is freed.
            if constexpr (CG == 2) tc_commit_pair(mma_done_bar);
            else tc_commit(mma_done_bar);
            drain_wait(mma_done_bar, 0);
        }
    } else {
        // ------------------------------------------------ epilogue
        const uint32_t ew = warp - 2u;                // epilogue warp 0..7
        const uint32_t quad = warp & 3u;              // TMEM lane quadrant of this warp
        const uint32_t half = ew >> 2;                // column half of the tile
        const uint32_t lane_row = quad * 32u + lane;  // query row within the tile
        constexpr uint32_t kHalfCols = BN / 2;
        constexpr uint32_t kChunks = kHalfCols / 32;
        uint32_t* hist = reinterpret_cast<uint32_t*>(smem + Cfg::kHistOffset + ew * Cfg::kWarpScratchBytes);
        uint32_t* const stage_row = hist + lane * kStageStride;
        float* xs = reinterpret_cast<float*>(smem + Cfg::kNormOffset) + ew * kHalfCols;
        uint2* const lists = p.cand + (static_cast<size_t>(blockIdx.x) * 2u + half) * kTileM * p.cap;
        uint2* const my_list = lists + static_cast<size_t>(lane_row) * p.cap;
        const uint32_t lane_base = (quad * 32u) << 16;
        uint32_t tile_iter = 0;
        bool ok = true;
        // Rank 0's accumulator-free barrier, released by both CTAs' epilogues.
        const uint32_t tempty_remote0 = CG == 2 ? mapa_shared(tempty_bar(0), 0) : 0u;
        const uint32_t tempty_remote1 = CG == 2 ? mapa_shared(tempty_bar(1), 0) : 0u;
        for (uint32_t unit = group; ok && unit < num_units; unit += groups) {
            const uint32_t qt = unit % p.n_qt, sp = unit / p.n_qt;
            const uint32_t bt0 = static_cast<uint32_t>((uint64_t)sp * p.n_bt / p.splits);
            const uint32_t bt1 = static_cast<uint32_t>((uint64_t)(sp + 1) * p.n_bt / p.splits);
            const uint32_t q = qt * kGroupM + rank * kTileM + lane_row;
            const bool qvalid = q < p.nq;
            float qn = 0.0f;
            if constexpr (METRIC == kEuclidean) {
                if (qvalid) qn = p.query_norms[q];
            }
            float tau = __int_as_float(0x7f800000);  // +inf: this list's own k-th key
            uint32_t cnt = 0;
            // The shared bound is read one tile ahead: the bound array may sit
            // in another GPU's memory, and a stale bound is still a valid one.
            uint32_t next_bound = qvalid ? __ldcg(p.qtau + q) : 0xFFFFFFFFu;
            for (uint32_t bt = bt0; bt < bt1; ++bt, ++tile_iter) {
                const uint32_t acc = tile_iter & 1u;
                const uint32_t acc_phase = (tile_iter >> 1) & 1u;
                const uint32_t bound = next_bound;
                if (qvalid && bt + 1 < bt1) next_bound = __ldcg(p.qtau + q);
                float thr = admission_threshold(tau, bound);
                const Admission<KIND, METRIC> adm_test(thr, qn);
                const uint32_t col0 = half * kHalfCols;
                const uint32_t row_half = bt * BN + col0;
                if constexpr (METRIC == kEuclidean) {
                    // stage this half-tile's base norms (rows past n read as 0)
                    for (uint32_t j = lane; j < kHalfCols; j += 32) {
                        const uint32_t r = row_half + j;
                        xs[j] = r < p.n ? __ldg(p.base_norms + r) : 0.0f;
                    }
                    __syncwarp();
                }
                ok = mbar_wait(tfull_bar(acc), acc_phase, abort_flag);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc_fence_after();
#pragma unroll 1
                for (uint32_t c = 0; c < kChunks; ++c) {
                    uint32_t v[32];
                    // tcgen05.ld is .sync.aligned: the warp must arrive converged.
                    __syncwarp();
                    tmem_ld_32x32b_x32(tmem_base + lane_base + acc * BN + col0 + c * 32u, v);
                    tmem_wait_ld();
                    if (c == kChunks - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            if constexpr (CG == 2) mbar_arrive_cluster(acc ? tempty_remote1 : tempty_remote0);
                            else mbar_arrive(tempty_bar(acc));
                        }
                    }
                    const uint32_t row0 = row_half + c * 32u;
                    if (row0 >= p.n) continue;
                    const uint32_t valid_rows = min(32u, p.n - row0);
                    uint32_t mword = valid_rows == 32u ? 0xFFFFFFFFu : ((1u << valid_rows) - 1u);
                    if (p.mask != nullptr) mword &= __ldg(p.mask + (row0 >> 5));
                    if (p.live != nullptr) mword &= __ldg(p.live + (row0 >> 5));
                    if (!qvalid) mword = 0;
                    const float* xn = xs + c * 32u;
                    // Admission mask, one compare per column; admitted columns
                    // are few, so only they are visited: a lane with any
                    // stages its half-chunk in shared memory and walks the set
                    // bits with the exact key test.
                    uint32_t am[4] = {0u, 0u, 0u, 0u};  // four independent chains
#pragma unroll
                    for (uint32_t i = 0; i < 32; ++i) am[i & 3u] |= adm_test.pass(v[i], xn[i]) ? (1u << i) : 0u;
                    const uint32_t adm = ((am[0] | am[1]) | (am[2] | am[3])) & mword;
                    if (__any_sync(0xffffffffu, adm != 0u)) {
#pragma unroll
                        for (uint32_t h = 0; h < 2; ++h) {
                            uint32_t hm = (adm >> (16u * h)) & 0xFFFFu;
                            if (__any_sync(0xffffffffu, __popc(hm) > 4)) {
                                // Many admissions (no tight bound yet): predicated
                                // appends over the half-chunk's 16 registers.
#pragma unroll
                                for (uint32_t j = 0; j < 16; ++j) {
                                    const uint32_t col = 16u * h + j;
                                    const float key = key_of<KIND, METRIC>(v[col], xn[col], qn);
                                    const bool take = ((hm >> j) & 1u) && key < thr;
                                    st_global_pred(my_list + cnt, __float_as_uint(key), p.row_offset + row0 + col, take);
                                    cnt += take ? 1u : 0u;
                                }
                            } else if (hm != 0u) {
                                // Few admissions: stage the half-chunk in shared
                                // memory and visit only the set bits, two per step.
#pragma unroll
                                for (uint32_t j = 0; j < 4; ++j)
                                    *reinterpret_cast<uint4*>(stage_row + 4u * j) =
                                        make_uint4(v[16u * h + 4u * j], v[16u * h + 4u * j + 1u],
                                                   v[16u * h + 4u * j + 2u], v[16u * h + 4u * j + 3u]);
                                do {
                                    const uint32_t i0 = __ffs(hm) - 1u;
                                    hm &= hm - 1u;
                                    const bool two = hm != 0u;
                                    const uint32_t i1 = two ? __ffs(hm) - 1u : i0;
                                    hm &= hm - 1u;
                                    const float k0 = key_of<KIND, METRIC>(stage_row[i0], xn[16u * h + i0], qn);
                                    const float k1 = key_of<KIND, METRIC>(stage_row[i1], xn[16u * h + i1], qn);
                                    const bool t0 = k0 < thr, t1 = two && k1 < thr;
                                    if (t0) my_list[cnt] = make_uint2(__float_as_uint(k0), p.row_offset + row0 + 16u * h + i0);
                                    cnt += t0 ? 1u : 0u;
                                    if (t1) my_list[cnt] = make_uint2(__float_as_uint(k1), p.row_offset + row0 + 16u * h + i1);
                                    cnt += t1 ? 1u : 0u;
                                } while (hm != 0u);
                            }
                        }
                    }
                }
                // Keep room for one more half-tile: compact any list that could
                // overflow, and a list not yet compacted in this unit once it
                // holds more than `early` entries, which gives it a threshold
                // (its k-th key) long before it would otherwise fill.
                __syncwarp();
                const bool first = p.early != 0u && cnt > p.early && tau == __int_as_float(0x7f800000);
                uint32_t need = __ballot_sync(0xffffffffu, cnt + kHalfCols > p.cap || first);
                while (need) {
                    const uint32_t L = __ffs(need) - 1;
                    const uint32_t cnt_l = __shfl_sync(0xffffffffu, cnt, L);
                    uint2* list_l = lists + static_cast<size_t>(quad * 32u + L) * p.cap;
                    const float th = compact_one(list_l, cnt_l, p.k, p.cap, hist);
                    if (lane == L) {
                        tau = th;
                        cnt = p.k;
                        atomicMin(p.qtau + q, ordered_key(th));
                    }
                    need &= need - 1;
                }
                if constexpr (METRIC == kEuclidean) __syncwarp();
            }
            if (!ok) break;
            // End of unit: reduce every list longer than its slot to its k
            // best, then publish (slot > k leaves short lists to the merge).
            __syncwarp();
            uint32_t need = __ballot_sync(0xffffffffu, cnt > p.slot);
            while (need) {
                const uint32_t L = __ffs(need) - 1;
                const uint32_t cnt_l = __shfl_sync(0xffffffffu, cnt, L);
                uint2* list_l = lists + static_cast<size_t>(quad * 32u + L) * p.cap;
                const float th = compact_one(list_l, cnt_l, p.k, p.cap, hist);
                if (lane == L) {
                    cnt = p.k;
                    atomicMin(p.qtau + q, ordered_key(th));
                }
                need &= need - 1;
            }
            __syncwarp();
            if (qvalid) {
                uint2* out = p.partial + ((static_cast<size_t>(q) * p.splits + sp) * 2u + half) * p.slot;
                const uint2 none = make_uint2(0x7f800000u, 0xFFFFFFFFu);
                if ((p.slot & 1u) == 0u) {
                    // slot even: both the list (cap entries, cap a multiple of
                    // 32) and this slot start on 16 bytes; two entries per access.
                    const uint4* src = reinterpret_cast<const uint4*>(my_list);
                    uint4* dst = reinterpret_cast<uint4*>(out);
                    for (uint32_t i = 0; i < p.slot / 2u; ++i) {
                        uint4 e = src[i];
                        if (2u * i >= cnt) e.x = none.x, e.y = none.y;
                        if (2u * i + 1u >= cnt) e.z = none.x, e.w = none.y;
                        dst[i] = e;
                    }
                } else {
                    for (uint32_t i = 0; i < p.slot; ++i) out[i] = i < cnt ? my_list[i] : none;
                }
            }
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    // Neither CTA of a pair leaves while the other may still signal its
    // barriers, read its shared memory (MMA) or land loads in it.
    if constexpr (CG == 2) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (CG == 2) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
        else tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

}  // namespace eb
