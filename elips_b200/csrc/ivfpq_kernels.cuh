// IVF-PQ search kernels, following GpuIVFPQIndex::search
// (src/gpu_engine/GpuIVFPQIndex.cpp:161-237):
//
//   1. probe: exact distances to every centroid + top-nprobe (the GpuPort
//      primitives in scan_kernels.cuh, as IvfIndexState::probe_lists,
//      src/gpu_engine/detail/IvfIndexState.cpp:395-423);
//   2. probe plan: the (query, probe slot) pairs are grouped by list
//      (count, plan, scatter), so that one CTA serves up to G queries that
//      probed the same list and reads the list's codes once for all of them;
//   3. ivfpq_group_scan_kernel: per (list, query group), a lookup table per
//      query [pq_dim][ksub] of the per-dimension terms of the reference's
//      decoded distance (decode_candidate_vector, GpuIVFPQIndex.cpp:132-148,
//      then elips::distance), summed per candidate subspace by subspace.
//      The terms are identical to the reference's, only their summation is
//      grouped by subspace; the approximate ranking only decides which
//      R = max(4k, k) candidates are reranked. Keeps the R best by
//      (approximate distance, slot) per (query, list);
//   4. the R-best merge across probed lists (merge_topk_kernel);
//   5. ivfpq_rerank_kernel: exact elips::distance on the raw vectors of the R
//      candidates, sequential fp32 (exact_rank, :37-71), top-k by
//      (distance, slot).
//
// Shared-memory layout of the lookup tables: the G queries of a group are
// packed in vectors of QP = min(G, 4) (one table entry holds the QP queries'
// values), so one vector load serves QP queries. The tables of the G / QP
// vector groups ("quads") are G / QP lanes apart and have a stride of
// pq_dim * ksub + 4 vectors (4 mod 8), which spreads the lanes that look up
// one candidate over distinct banks.
#pragma once

#include <cstdint>
#include <type_traits>

#include "ptx.cuh"
#include "scan_kernels.cuh"

namespace eb {

// ----------------------------------------------------------------- plan

constexpr uint32_t kPlanThreads = 1024;
constexpr uint32_t kPlanSortMax = 8192;  // lists visited largest first up to this many

// Whether list l (< nlist) is one this index owns: owned = null for all
// lists, else a bitmask (bit l & 31 of word l >> 5) of one GPU's share of a
// list-sharded index.
__device__ __forceinline__ bool ivf_owned(const uint32_t* owned, uint32_t l, uint32_t nlist) {
    return l < nlist && (owned == nullptr || ((owned[l >> 5] >> (l & 31u)) & 1u));
}

// pair = q * nprobe + p. Counts the pairs of every list this index owns; a
// pair whose list is not owned gets an empty candidate list.
static __global__ void ivf_pair_count_kernel(const uint32_t* __restrict__ probes, uint32_t npairs, uint32_t nlist,
                                             const uint32_t* __restrict__ owned, uint32_t* __restrict__ counts,
                                             uint2* __restrict__ partial, uint32_t r) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= npairs) return;
    const uint32_t l = probes[i];
    if (ivf_owned(owned, l, nlist)) {
        atomicAdd(&counts[l], 1u);
        return;
    }
    for (uint32_t j = 0; j < r; ++j) partial[static_cast<size_t>(i) * r + j] = make_uint2(0x7f800000u, 0xFFFFFFFFu);
}

// Exclusive scan over n values (whole block, chunks of blockDim.x): get(i)
// gives value i, put(i, prefix) receives its exclusive prefix. Returns the
// total. Ends with a barrier.
template <class Get, class Put>
__device__ uint32_t block_exclusive_scan(uint32_t n, Get get, Put put, uint32_t* warp_sums) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t carry = 0;
    for (uint32_t base = 0; base < n; base += blockDim.x) {
        const uint32_t i = base + threadIdx.x;
        const uint32_t v = i < n ? get(i) : 0u;
        uint32_t incl = v;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= static_cast<uint32_t>(off)) incl += t;
        }
        if (lane == 31) warp_sums[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const uint32_t w = lane < nw ? warp_sums[lane] : 0u;
            uint32_t wi = w;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, wi, off);
                if (lane >= static_cast<uint32_t>(off)) wi += t;
            }
            if (lane < nw) warp_sums[lane] = wi - w;
            if (lane == 31) warp_sums[32] = wi;
        }
        __syncthreads();
        if (i < n) put(i, carry + warp_sums[warp] + incl - v);
        carry += warp_sums[32];
        __syncthreads();
    }
    return carry;
}

// One CTA. list_start[l]: first pair of list l in the grouped pair array
// (lists in index order); items: one {list, first pair} per group of up to G
// pairs of one list, lists with the most members first (when at most
// kPlanSortMax lists; index order otherwise). ctrl[0] = item count,
// ctrl[1] = work-queue cursor (reset). cursor[] is reset for the scatter.
static __global__ void __launch_bounds__(kPlanThreads)
    ivf_group_plan_kernel(const uint32_t* __restrict__ counts, const uint32_t* __restrict__ list_off, uint32_t nlist,
                          uint32_t G, uint32_t* __restrict__ list_start, uint32_t* __restrict__ cursor,
                          uint2* __restrict__ items, uint32_t* __restrict__ ctrl) {
    extern __shared__ unsigned long long order[];
    __shared__ uint32_t warp_sums[33];
    const bool sorted = nlist <= kPlanSortMax;
    if (sorted) {
        uint32_t npow2 = 1;
        while (npow2 < nlist) npow2 <<= 1;
        for (uint32_t i = threadIdx.x; i < npow2; i += blockDim.x) {
            const uint32_t members = i < nlist ? list_off[i + 1] - list_off[i] : 0u;
            order[i] = i < nlist ? (static_cast<unsigned long long>(0xFFFFFFFFu - members) << 32) | i : ~0ull;
        }
        block_bitonic_sort(order, npow2);
    }
    block_exclusive_scan(
        nlist, [&](uint32_t l) { return counts[l]; },
        [&](uint32_t l, uint32_t pre) {
            list_start[l] = pre;
            cursor[l] = 0;
        },
        warp_sums);
    auto list_at = [&](uint32_t i) { return sorted ? static_cast<uint32_t>(order[i] & 0xFFFFFFFFu) : i; };
    const uint32_t total = block_exclusive_scan(
        nlist, [&](uint32_t i) { return (counts[list_at(i)] + G - 1) / G; },
        [&](uint32_t i, uint32_t pre) {
            const uint32_t l = list_at(i);
            const uint32_t groups = (counts[l] + G - 1) / G;
            for (uint32_t g = 0; g < groups; ++g) items[pre + g] = make_uint2(l, list_start[l] + g * G);
        },
        warp_sums);
    if (threadIdx.x == 0) {
        ctrl[0] = total;
        ctrl[1] = 0;
    }
}

static __global__ void ivf_pair_scatter_kernel(const uint32_t* __restrict__ probes, uint32_t npairs, uint32_t nlist,
                                               const uint32_t* __restrict__ owned,
                                               const uint32_t* __restrict__ list_start,
                                               uint32_t* __restrict__ cursor, uint32_t* __restrict__ pairs) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= npairs) return;
    const uint32_t l = probes[i];
    if (ivf_owned(owned, l, nlist)) pairs[list_start[l] + atomicAdd(&cursor[l], 1u)] = i;
}

// Gather position of each pair's first candidate: the candidates of a query
// are its probed lists' members in probe order, then member order
// (IvfIndexState::gather_candidates, IvfIndexState.cpp:466-504).
static __global__ void ivf_pair_offsets_kernel(const uint32_t* __restrict__ probes, uint32_t nq, uint32_t nprobe,
                                               uint32_t nlist, const uint32_t* __restrict__ list_off,
                                               uint32_t* __restrict__ pair_off) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    uint32_t at = 0;
    for (uint32_t i = 0; i < nprobe; ++i) {
        const size_t pair = static_cast<size_t>(q) * nprobe + i;
        pair_off[pair] = at;
        const uint32_t l = probes[pair];
        if (l < nlist) at += list_off[l + 1] - list_off[l];
    }
}

// rows[q][i]: gather position -> slot (the probed list holding it, then the
// member at that offset). -1 stays -1.
static __global__ void ivf_gather_to_slot_kernel(int64_t* __restrict__ rows, uint32_t nq, uint32_t k,
                                                 const uint32_t* __restrict__ probes, uint32_t nprobe,
                                                 const uint32_t* __restrict__ pair_off,
                                                 const uint32_t* __restrict__ list_off,
                                                 const uint32_t* __restrict__ list_rows) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<uint64_t>(nq) * k) return;
    const int64_t gp = rows[t];
    if (gp < 0) return;
    const uint32_t q = static_cast<uint32_t>(t / k);
    const uint32_t* off = pair_off + static_cast<size_t>(q) * nprobe;
    uint32_t lo = 0, hi = nprobe - 1;  // largest i with off[i] <= gp (that list holds gp)
    while (lo < hi) {
        const uint32_t mid = (lo + hi + 1) / 2;
        if (off[mid] <= static_cast<uint64_t>(gp)) lo = mid;
        else hi = mid - 1;
    }
    const uint32_t l = probes[static_cast<size_t>(q) * nprobe + lo];
    rows[t] = list_rows[list_off[l] + static_cast<uint32_t>(gp - off[lo])];
}

// ----------------------------------------------------------------- scan

constexpr uint32_t kGroupWarps = 16;
constexpr uint32_t kGroupThreads = kGroupWarps * 32;

// Candidates of one list each query of a group sees per round (between two
// block barriers), for G queries per group.
__host__ __device__ constexpr uint32_t group_round(uint32_t) { return 1024u; }

// Queries per lane (one vector table lookup serves them all).
__host__ __device__ constexpr uint32_t group_qp(uint32_t G) { return G < 4u ? G : 4u; }

// Vectors between the tables of two quads.
__host__ __device__ constexpr uint32_t group_lut_stride(uint32_t m, uint32_t ksub) { return m * ksub + 4u; }

// Per-query candidate buffer: the R kept plus room for a round of appends,
// with slack so that compactions are rare.
__host__ __device__ constexpr uint32_t group_capacity(uint32_t G, uint32_t r) {
    return ((r + 256u > 2u * r ? r + 256u : 2u * r) + group_round(G) + 31u) / 32u * 32u;
}

struct GroupLayout {
    uint32_t lut, qv, cv, buf, hist, cnt, thr, bound, item, total;
};

__host__ __device__ inline GroupLayout group_layout(uint32_t G, uint32_t d, uint32_t lut_stride, uint32_t capq) {
    auto up16 = [](uint32_t x) { return (x + 15u) / 16u * 16u; };
    GroupLayout L{};
    uint32_t o = 0;
    L.lut = o;
    o = up16(o + G * lut_stride * 4u);
    L.qv = o;
    o = up16(o + G * d * 4u);
    L.cv = o;
    o = up16(o + d * 4u);
    L.buf = o;
    o = up16(o + G * capq * 8u);
    L.hist = o;
    o = up16(o + G * 256u * 4u);
    L.cnt = o;
    o = up16(o + G * 4u);
    L.thr = o;
    o = up16(o + 2u * G * 4u);
    L.bound = o;
    o = up16(o + 2u * G * 4u);
    L.item = o;
    o = up16(o + 16u);
    L.total = o;
    return L;
}

struct IvfGroupParams {
    const float* queries;       // [nq][d]
    const float* centroids;     // [nlist][d]
    const float* codebook;      // [m][ksub][sub]
    const uint8_t* list_codes;  // [n][m], list-major
    const uint32_t* list_rows;  // [n] slot of each list-major position
    const uint32_t* list_off;   // [nlist + 1]
    const uint32_t* counts;     // [nlist] pairs per list
    const uint32_t* list_start; // [nlist] first pair of each list in `pairs`
    const uint32_t* pairs;      // pair ids grouped by list
    const uint2* items;         // {list, first pair}
    uint32_t* ctrl;             // [0] item count, [1] work-queue cursor
    uint2* partial;             // [npairs][r] {key bits, slot (PQ) or gather position (flat)}
    uint32_t* qbound;           // [nq] ordered key: the query's R-th best so far, over all lists
    const float* list_vecs;     // flat: [n][d] raw rows, list-major
    const uint32_t* pair_off;   // flat: [npairs] gather position of the pair's first member
    uint32_t d, nprobe, m, pq_bits, r, capq, lut_stride;
    int metric;
};

// Reduces buf[0, n) (n > r) in place to its r smallest composites
// (ordered key << 32 | slot; unique, slots are unique) and returns the
// ordered key of the r-th. One warp; hist is 256 words of its own.
static __device__ __noinline__ uint32_t warp_select_compact(uint2* buf, uint32_t n, uint32_t r, uint32_t* hist) {
    const uint32_t lane = threadIdx.x & 31u;
    unsigned long long prefix = 0, pmask = 0;
    uint32_t rank = r;
    for (int pass = 0; pass < 8; ++pass) {
        const uint32_t shift = 56u - 8u * static_cast<uint32_t>(pass);
        for (uint32_t b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
        for (uint32_t j = lane; j < n; j += 32) {
            const unsigned long long c = composite_of(buf[j]);
            if ((c & pmask) == prefix) atomicAdd(&hist[(c >> shift) & 255u], 1u);
        }
        __syncwarp();
        uint32_t bins[8], local = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            bins[i] = hist[lane * 8 + i];
            local += bins[i];
        }
        uint32_t incl = local;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= static_cast<uint32_t>(off)) incl += t;
        }
        const uint32_t excl = incl - local;
        const bool mine = excl < rank && rank <= incl;
        const uint32_t owner = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
        uint32_t digit = 0, before = 0, inbin = 0;
        if (mine) {
            uint32_t acc = excl;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (inbin == 0 && acc + bins[i] >= rank) {
                    digit = lane * 8 + i;
                    before = acc;
                    inbin = bins[i];
                }
                acc += bins[i];
            }
        }
        digit = __shfl_sync(0xffffffffu, digit, owner);
        before = __shfl_sync(0xffffffffu, before, owner);
        inbin = __shfl_sync(0xffffffffu, inbin, owner);
        rank -= before;
        prefix |= static_cast<unsigned long long>(digit) << shift;
        pmask |= 255ull << shift;
        __syncwarp();
        if (pass == 3 && inbin == rank) {  // every candidate with the r-th key is kept
            prefix |= 0xFFFFFFFFull;
            break;
        }
    }
    uint32_t out = 0;
    for (uint32_t base = 0; base < n; base += 32) {
        const uint32_t j = base + lane;
        const uint2 e = j < n ? buf[j] : make_uint2(0u, 0u);
        const bool keep = j < n && composite_of(e) <= prefix;
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        __syncwarp();
        if (keep) buf[out + __popc(bal & lanemask_lt())] = e;
        out += __popc(bal);
        __syncwarp();
    }
    return static_cast<uint32_t>(prefix >> 32);
}

// Lookup tables of the group: the value for query g and codeword (s, c) is
// at float index ((g / QP) * lut_stride + s * ksub + c) * QP + g % QP: the
// subspace-s terms of query g against centroid + codeword (s, c), summed over
// the subspace's dimensions in order. A thread computes 4 entries of one
// subspace, so each query value it loads serves 4 entries.
template <int G>
__device__ __forceinline__ void build_group_lut(float* lut, uint32_t lut_stride, const float* qv, const float* cv,
                                                const float* __restrict__ codebook, uint32_t d, uint32_t m,
                                                uint32_t bits, uint32_t ng, int metric) {
    constexpr uint32_t CL = 4;
    constexpr uint32_t QP = group_qp(G);
    const uint32_t sub = d / m, ksub = 1u << bits, per_s = ksub / CL, units = m * per_s;
    for (uint32_t u = threadIdx.x; u < units; u += blockDim.x) {
        const uint32_t s = u / per_s, c0 = u - s * per_s;
        const float* cs = cv + s * sub;
        const float* qs = qv + s * sub;
        const float* cw[CL];
#pragma unroll
        for (uint32_t i = 0; i < CL; ++i) cw[i] = codebook + static_cast<size_t>(s * ksub + c0 + i * per_s) * sub;
        float acc[CL][G];
#pragma unroll
        for (uint32_t i = 0; i < CL; ++i)
#pragma unroll
            for (int g = 0; g < G; ++g) acc[i][g] = 0.0f;
        auto step = [&](uint32_t t, const float (&w)[CL]) {
            const float cst = cs[t];
            float qx[G];
#pragma unroll
            for (int g = 0; g < G; ++g) qx[g] = qs[g * d + t];
#pragma unroll
            for (uint32_t i = 0; i < CL; ++i) {
                const float dv = __fadd_rn(cst, w[i]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    if (metric == kMetricL2) {
                        const float df = __fsub_rn(qx[g], dv);
                        acc[i][g] = __fadd_rn(acc[i][g], __fmul_rn(df, df));
                    } else {
                        acc[i][g] = __fadd_rn(acc[i][g], __fmul_rn(qx[g], dv));
                    }
                }
            }
        };
        if ((sub & 3u) == 0) {
            for (uint32_t t = 0; t < sub; t += 4) {
                float4 w4[CL];
#pragma unroll
                for (uint32_t i = 0; i < CL; ++i) w4[i] = __ldg(reinterpret_cast<const float4*>(cw[i] + t));
                float w[CL];
#pragma unroll
                for (uint32_t i = 0; i < CL; ++i) w[i] = w4[i].x;
                step(t, w);
#pragma unroll
                for (uint32_t i = 0; i < CL; ++i) w[i] = w4[i].y;
                step(t + 1, w);
#pragma unroll
                for (uint32_t i = 0; i < CL; ++i) w[i] = w4[i].z;
                step(t + 2, w);
#pragma unroll
                for (uint32_t i = 0; i < CL; ++i) w[i] = w4[i].w;
                step(t + 3, w);
            }
        } else {
            for (uint32_t t = 0; t < sub; ++t) {
                float w[CL];
#pragma unroll
                for (uint32_t i = 0; i < CL; ++i) w[i] = __ldg(cw[i] + t);
                step(t, w);
            }
        }
        (void)ng;  // entries of absent queries hold the terms of a zero query; never read
#pragma unroll
        for (uint32_t i = 0; i < CL; ++i) {
            const uint32_t e = s * ksub + c0 + i * per_s;
#pragma unroll
            for (uint32_t q = 0; q < G / QP; ++q) {
                float* dst = lut + (static_cast<size_t>(q) * lut_stride + e) * QP;
                if constexpr (QP == 4) {
                    *reinterpret_cast<float4*>(dst) =
                        make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
                } else if constexpr (QP == 2) {
                    *reinterpret_cast<float2*>(dst) = make_float2(acc[i][2 * q], acc[i][2 * q + 1]);
                } else {
                    dst[0] = acc[i][q];
                }
            }
        }
    }
}

// Approximate key of a candidate from its summed table entries.
__device__ __forceinline__ float group_key(int metric, float sum) {
    return metric == kMetricL2 ? sqrtf(sum) : finish_dot(metric, sum);
}

// Sums are compared in a "z" domain that is monotone in the key: the ordered
// sum for L2 (key = sqrt(sum) rises with it), its complement for the inner
// products (key = 1 - sum or -sum falls as it rises).
__device__ __forceinline__ uint32_t group_z(int metric, float sum) {
    const uint32_t o = ordered_key(sum);
    return metric == kMetricL2 ? o : ~o;
}

// Admission bound in the z domain: the smallest z whose key's ordered value
// reaches T (so ordered(key) < T exactly when z < bound). One warp, a 32-way
// search over the z values of non-NaN sums (L2 sums are never below +0):
// [ordered(+0), ordered(+inf)] for L2, [~ordered(+inf), ~ordered(-inf)] for
// the inner products. 0xFFFFFFFF when no finite or infinite sum reaches T.
static __device__ __noinline__ uint32_t warp_sum_bound(uint32_t T, int metric) {
    const uint32_t lane = threadIdx.x & 31u;
    auto reaches = [&](uint64_t z) {
        const uint32_t o = metric == kMetricL2 ? static_cast<uint32_t>(z) : ~static_cast<uint32_t>(z);
        return ordered_key(group_key(metric, key_to_float(o))) >= T;
    };
    uint64_t lo = metric == kMetricL2 ? 0x80000000ull : 0x007FFFFFull, hi = 0xFF800000ull;
    if (!__shfl_sync(0xffffffffu, reaches(hi), 0)) return 0xFFFFFFFFu;
    // invariant: reaches(hi), and no z below lo in the range reaches T
    while (hi - lo > 31) {
        const uint64_t step = (hi - lo) / 33 > 0 ? (hi - lo) / 33 : 1ull;
        const uint64_t z = lo + step * (lane + 1);
        const uint32_t bal = __ballot_sync(0xffffffffu, reaches(z));
        if (bal == 0) {
            lo = lo + step * 32 + 1;
        } else {
            const uint32_t f = __ffs(bal) - 1;
            hi = lo + step * (f + 1);
            if (f > 0) lo = lo + step * f + 1;
        }
    }
    const uint64_t z = lo + lane;
    const uint32_t bal = __ballot_sync(0xffffffffu, z <= hi && reaches(z));
    return static_cast<uint32_t>(lo + (__ffs(bal) - 1));
}

// QP consecutive floats from shared memory (one scalar or vector load).
template <uint32_t QP>
__device__ __forceinline__ void lds_vec(uint32_t addr, float (&v)[QP]) {
    if constexpr (QP == 4) {
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                     : "r"(addr));
    } else if constexpr (QP == 2) {
        asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v[0]), "=f"(v[1]) : "r"(addr));
    } else {
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v[0]) : "r"(addr));
    }
}

// Code words of one candidate in registers (MB = code bytes: 4, 8, 16, 32;
// MB = 0 keeps none and reads the bytes at lookup time).
template <int MB>
struct CodeWords {
    uint32_t w[MB >= 4 ? MB / 4 : 1];
};

template <int MB>
__device__ __forceinline__ CodeWords<MB> load_code(const uint8_t* __restrict__ codes, uint32_t pos, bool in) {
    CodeWords<MB> c;
    if constexpr (MB >= 16) {
#pragma unroll
        for (int v = 0; v < MB / 16; ++v) {
            const uint4 x = in ? __ldg(reinterpret_cast<const uint4*>(codes + static_cast<size_t>(pos) * MB) + v)
                               : make_uint4(0u, 0u, 0u, 0u);
            c.w[4 * v] = x.x;
            c.w[4 * v + 1] = x.y;
            c.w[4 * v + 2] = x.z;
            c.w[4 * v + 3] = x.w;
        }
    } else if constexpr (MB == 8) {
        const uint2 x = in ? __ldg(reinterpret_cast<const uint2*>(codes + static_cast<size_t>(pos) * 8)) : make_uint2(0u, 0u);
        c.w[0] = x.x;
        c.w[1] = x.y;
    } else if constexpr (MB == 4) {
        c.w[0] = in ? __ldg(reinterpret_cast<const uint32_t*>(codes + static_cast<size_t>(pos) * 4)) : 0u;
    } else {
        c.w[0] = 0u;
    }
    return c;
}

// Exact elips::distance sums of one raw row against the G queries of the
// group (Metrics.cpp:20-37: sequential over dimensions, no FMA).
template <int G>
__device__ __forceinline__ void flat_sums(const float* __restrict__ x, const float* qv, uint32_t d, bool l2,
                                          float (&acc)[G]) {
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.0f;
    auto term = [&](uint32_t t, float xv, const float (&qx)[G]) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (l2) {
                const float df = __fsub_rn(qx[g], xv);
                acc[g] = __fadd_rn(acc[g], __fmul_rn(df, df));
            } else {
                acc[g] = __fadd_rn(acc[g], __fmul_rn(qx[g], xv));
            }
        }
        (void)t;
    };
    if ((d & 3u) == 0) {
        for (uint32_t t = 0; t < d; t += 4) {
            const float4 xv = __ldg(reinterpret_cast<const float4*>(x + t));
            float4 q4[G];
#pragma unroll
            for (int g = 0; g < G; ++g) q4[g] = *reinterpret_cast<const float4*>(qv + g * d + t);
            float qx[G];
#pragma unroll
            for (int g = 0; g < G; ++g) qx[g] = q4[g].x;
            term(t, xv.x, qx);
#pragma unroll
            for (int g = 0; g < G; ++g) qx[g] = q4[g].y;
            term(t + 1, xv.y, qx);
#pragma unroll
            for (int g = 0; g < G; ++g) qx[g] = q4[g].z;
            term(t + 2, xv.z, qx);
#pragma unroll
            for (int g = 0; g < G; ++g) qx[g] = q4[g].w;
            term(t + 3, xv.w, qx);
        }
    } else {
        for (uint32_t t = 0; t < d; ++t) {
            float qx[G];
#pragma unroll
            for (int g = 0; g < G; ++g) qx[g] = qv[g * d + t];
            term(t, __ldg(x + t), qx);
        }
    }
}

// Persistent CTAs over the plan's items (a work queue). Per item: list l and
// up to G of its pairs. Each query of the group keeps its R best candidates
// of the list by (approximate key, slot) in a shared-memory buffer:
//   * a candidate is appended when its key is below the list's own bound
//     (the R-th kept key, strict: candidates come in ascending slot order, so
//     a later equal key ranks after the kept one) and not above the query's
//     bound over all its lists (qbound: the R-th key of some list, so at least
//     R candidates of the query are at or below it);
//   * the test runs on the raw sum against the bound carried into the sum's
//     z domain (warp_sum_bound), the key is computed for appended ones only;
//   * at a round boundary a buffer that could overflow is compacted to R by
//     one warp, and the bounds are refreshed.
//
// FLAT = true scores exact distances on the raw rows instead (IVF-Flat,
// GpuIVFFlatIndex.cpp:44-103): a lane computes one candidate for all G
// queries, and the id kept is the candidate's gather position, which orders
// ties as the reference's top_k over the gathered candidates does.
template <int G, int MB, int BITS, bool FLAT>
__global__ void __launch_bounds__(kGroupThreads, 1) ivfpq_group_scan_kernel(const IvfGroupParams p) {
    constexpr uint32_t QP = FLAT ? G : group_qp(G);    // queries per lane
    constexpr uint32_t P = G / QP;                      // lanes per candidate
    constexpr uint32_t kCpi = 32u / P;                  // candidates per warp step
    constexpr uint32_t kRound = group_round(G);         // candidates per round
    constexpr uint32_t kSteps = kRound / (kGroupWarps * kCpi);
    static_assert(kSteps * QP <= 32, "admission mask is 32 bits");
    extern __shared__ __align__(16) uint8_t smem[];
    const GroupLayout L = group_layout(G, p.d, p.lut_stride, p.capq);
    float* lut = reinterpret_cast<float*>(smem + L.lut);
    float* qv = reinterpret_cast<float*>(smem + L.qv);
    float* cv = reinterpret_cast<float*>(smem + L.cv);
    uint2* buf = reinterpret_cast<uint2*>(smem + L.buf);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + L.hist);
    uint32_t* s_cnt = reinterpret_cast<uint32_t*>(smem + L.cnt);
    uint32_t* s_thr = reinterpret_cast<uint32_t*>(smem + L.thr);      // [G] list bound, [G] applied T
    uint32_t* s_bound = reinterpret_cast<uint32_t*>(smem + L.bound);  // [G] z bound, [G] query ids
    uint32_t* s_item = reinterpret_cast<uint32_t*>(smem + L.item);    // next item: live, list, first, ng
    __shared__ uint32_t s_pairoff[G];                                 // flat: gather offset of each pair
    // Round barrier, split in two: a warp arrives when its appends of round g
    // are done and waits for the others only before appending in round g + 1,
    // so its lookups of round g + 1 overlap the slower warps' round g.
    __shared__ __align__(8) uint64_t s_rbar;
    __shared__ uint32_t s_need[2];   // [g & 1] = g: an append of round g left a buffer short of a round's room
    __shared__ int s_abort;

    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t pq = lane % P, j = lane / P;  // this lane: quad pq of candidate j
    uint32_t qmask = 0;                          // lanes of the same quad
#pragma unroll
    for (uint32_t jj = 0; jj < kCpi; ++jj) qmask |= 1u << (jj * P + pq);
    const uint32_t kmask = (1u << p.pq_bits) - 1u;
    const uint32_t lut_q = smem_u32(lut) + pq * p.lut_stride * QP * 4u;  // this quad's tables

    // Warp w (< ng) refreshes query w's z bound from its list bound and the
    // query's global bound qb; recomputed only when the combined bound moved.
    // No barrier guards it: readers see the old or the new bound, both valid.
    auto refresh_bound = [&](uint32_t w, uint32_t qb) {
        const uint32_t T = min(s_thr[w], qb == 0xFFFFFFFFu ? qb : qb + 1u);
        if (T != s_thr[G + w]) {
            const uint32_t b = warp_sum_bound(T, p.metric);
            if (lane == 0) {
                s_thr[G + w] = T;
                s_bound[w] = b;
            }
        }
    };
    // Thread 0 takes the next item off the work queue into s_item.
    auto fetch_item = [&]() {
        const uint32_t it = atomicAdd(&p.ctrl[1], 1u);
        const bool live = it < p.ctrl[0];
        uint32_t list = 0, first = 0, ng = 0;
        if (live) {
            const uint2 item = p.items[it];
            list = item.x;
            first = item.y;
            ng = min(static_cast<uint32_t>(G), p.list_start[list] + p.counts[list] - first);
        }
        s_item[0] = live ? 1u : 0u;
        s_item[1] = list;
        s_item[2] = first;
        s_item[3] = ng;
    };

    const uint32_t rbar = smem_u32(&s_rbar);
    if (tid == 0) {
        mbar_init(rbar, kGroupWarps);
        s_need[0] = s_need[1] = 0xFFFFFFFFu;
        s_abort = 0;
        fetch_item();
    }
    __syncthreads();
    uint32_t g = 0;  // rounds so far (the same count in every warp)
    for (;;) {
        if (s_item[0] == 0) break;
        const uint32_t list = s_item[1], first = s_item[2], ng = s_item[3];
        for (uint32_t i = tid; i < G * p.d; i += blockDim.x) {
            const uint32_t gg = i / p.d, t = i - gg * p.d;
            qv[i] = gg < ng ? p.queries[static_cast<size_t>(p.pairs[first + gg] / p.nprobe) * p.d + t] : 0.0f;
        }
        for (uint32_t i = tid; i < p.d; i += blockDim.x) cv[i] = p.centroids[static_cast<size_t>(list) * p.d + i];
        if (tid < G) {
            s_cnt[tid] = 0;
            s_thr[tid] = 0xFFFFFFFFu;
            s_thr[G + tid] = 0xFFFFFFFFu;
            s_bound[tid] = 0xFFFFFFFFu;
            s_bound[G + tid] = tid < ng ? p.pairs[first + tid] / p.nprobe : 0u;
            if constexpr (FLAT) s_pairoff[tid] = tid < ng ? p.pair_off[p.pairs[first + tid]] : 0u;
        }
        __syncthreads();
        // The query's bound (possibly another GPU's memory) is loaded before
        // the lookup tables are built and applied after.
        const uint32_t qb0 = warp < ng ? p.qbound[s_bound[G + warp]] : 0u;
        if constexpr (!FLAT) {
            build_group_lut<G>(lut, p.lut_stride, qv, cv, p.codebook, p.d, p.m, p.pq_bits, ng, p.metric);
        }
        if (warp < ng) refresh_bound(warp, qb0);
        if constexpr (!FLAT) __syncthreads();

        const uint32_t b0 = p.list_off[list], b1 = p.list_off[list + 1];
        bool qvalid[QP];
#pragma unroll
        for (uint32_t qi = 0; qi < QP; ++qi) qvalid[qi] = pq * QP + qi < ng;
        // L1 prefetch of the code lines one round ahead (the first round's now)
        auto prefetch_round = [&](uint32_t start) {
            if constexpr (!FLAT) {
                const uint32_t round_lines = (kRound * p.m + 127u) / 128u;
                if (tid < round_lines && start < b1) {
                    const uint8_t* a = p.list_codes + static_cast<size_t>(start) * p.m + tid * 128u;
                    if (a < p.list_codes + static_cast<size_t>(b1) * p.m)
                        asm volatile("prefetch.global.L1 [%0];" ::"l"(a));
                }
            }
        };
        prefetch_round(b0);
        // The rounds, for L2 (admission on the raw non-negative sum's bits) or
        // the inner products (on the complemented ordered sum).
        auto scan_rounds = [&](auto l2_tag) {
            constexpr bool kL2 = decltype(l2_tag)::value;
            for (uint32_t base = b0; base < b1; base += kRound) {
                uint32_t zb[QP];
#pragma unroll
                for (uint32_t qi = 0; qi < QP; ++qi) {
                    const uint32_t z = s_bound[pq * QP + qi];
                    zb[qi] = kL2 ? (z >= 0x80000000u ? z - 0x80000000u : 0u) : z;
                }
                const uint32_t qb = warp < ng ? p.qbound[s_bound[G + warp]] : 0u;
                prefetch_round(base + kRound);
                CodeWords<MB> cur[FLAT ? 1 : kSteps];
                if constexpr (!FLAT) {
#pragma unroll
                    for (uint32_t st = 0; st < kSteps; ++st) {
                        const uint32_t pos = base + (st * kGroupWarps + warp) * kCpi + j;
                        cur[st] = load_code<MB>(p.list_codes, pos, pos < b1);
                    }
                } else {
                    (void)cur;
                }
                float sums[kSteps][QP];
#pragma unroll
                for (uint32_t st = 0; st < kSteps; ++st)
#pragma unroll
                    for (uint32_t qi = 0; qi < QP; ++qi) sums[st][qi] = 0.0f;
                if constexpr (FLAT) {
#pragma unroll
                    for (uint32_t st = 0; st < kSteps; ++st) {
                        const uint32_t pos = base + (st * kGroupWarps + warp) * kCpi + j;
                        if (pos < b1) flat_sums<G>(p.list_vecs + static_cast<size_t>(pos) * p.d, qv, p.d, kL2, sums[st]);
                    }
                } else if constexpr (MB >= 4) {
                    // subspace-major over the round's steps: independent chains,
                    // each summed in subspace order
#pragma unroll
                    for (int sp = 0; sp < MB; ++sp) {
#pragma unroll
                        for (uint32_t st = 0; st < kSteps; ++st) {
                            const uint32_t byte = __byte_perm(cur[st].w[sp >> 2], 0u, 0x4440u + (sp & 3));
                            const uint32_t e = BITS == 8 ? static_cast<uint32_t>(sp) * 256u + byte
                                                         : (static_cast<uint32_t>(sp) << p.pq_bits) + (byte & kmask);
                            float v[QP];
                            lds_vec<QP>(lut_q + e * (QP * 4u), v);
#pragma unroll
                            for (uint32_t qi = 0; qi < QP; ++qi) sums[st][qi] = __fadd_rn(sums[st][qi], v[qi]);
                        }
                    }
                } else {
#pragma unroll
                    for (uint32_t st = 0; st < kSteps; ++st) {
                        const uint32_t pos = base + (st * kGroupWarps + warp) * kCpi + j;
                        const uint8_t* cp = p.list_codes + static_cast<size_t>(pos) * p.m;
                        for (uint32_t sp = 0; sp < p.m; ++sp) {
                            const uint32_t b = pos < b1 ? (static_cast<uint32_t>(__ldg(cp + sp)) & kmask) : 0u;
                            float v[QP];
                            lds_vec<QP>(lut_q + ((sp << p.pq_bits) + b) * (QP * 4u), v);
#pragma unroll
                            for (uint32_t qi = 0; qi < QP; ++qi) sums[st][qi] = __fadd_rn(sums[st][qi], v[qi]);
                        }
                    }
                }
                uint32_t amask = 0;  // bit st * QP + qi
#pragma unroll
                for (uint32_t st = 0; st < kSteps; ++st) {
                    const uint32_t pos = base + (st * kGroupWarps + warp) * kCpi + j;
#pragma unroll
                    for (uint32_t qi = 0; qi < QP; ++qi) {
                        const bool pass = kL2 ? __float_as_uint(sums[st][qi]) < zb[qi]
                                              : ~ordered_key(sums[st][qi]) < zb[qi];
                        if (pass && pos < b1 && qvalid[qi]) amask |= 1u << (st * QP + qi);
                    }
                }
                // Every warp's appends of the previous round are done (it
                // arrived after them); a warp that saw a buffer left with less
                // than a round of room stamped s_need with that round, so all
                // warps take the same decision: the short buffers are compacted
                // (one warp each) before anyone appends again. The stamp of
                // round g - 1 cannot be overwritten before every warp read it:
                // round g + 1's appends wait for every warp's round g arrival.
                ++g;
                if (g > 1) {
                    if (!mbar_wait_for(rbar, g & 1u, &s_abort, kWaitTimeoutCycles)) amask = 0;
                    if (s_need[(g - 1u) & 1u] == g - 1u) {
                        if (warp < ng && s_cnt[warp] + kRound > p.capq) {
                            const uint32_t t =
                                warp_select_compact(buf + warp * p.capq, s_cnt[warp], p.r, hist + warp * 256u);
                            if (lane == 0) {
                                s_cnt[warp] = p.r;
                                s_thr[warp] = t;
                                atomicMin(&p.qbound[s_bound[G + warp]], t);
                            }
                            __syncwarp();
                        }
                        __syncthreads();
                    }
                    if (warp < ng) refresh_bound(warp, qb);
                }
                const bool appended = __any_sync(0xffffffffu, amask != 0);
                bool need = false;  // some count this warp saw leaves less than a round of room
                if (appended) {
#pragma unroll
                    for (uint32_t st = 0; st < kSteps; ++st) {
#pragma unroll
                        for (uint32_t qi = 0; qi < QP; ++qi) {
                            const bool admit = (amask >> (st * QP + qi)) & 1u;
                            const uint32_t bal = __ballot_sync(0xffffffffu, admit) & qmask;
                            if (__any_sync(0xffffffffu, bal != 0)) {
                                const uint32_t gq = pq * QP + qi;
                                const uint32_t pos = base + (st * kGroupWarps + warp) * kCpi + j;
                                const uint32_t leader = bal ? __ffs(bal) - 1u : lane;
                                uint32_t at = 0;
                                if (admit && lane == leader) at = atomicAdd(&s_cnt[gq], static_cast<uint32_t>(__popc(bal)));
                                at = __shfl_sync(0xffffffffu, at, leader);
                                if (admit) {
                                    const uint32_t id = FLAT ? s_pairoff[gq] + (pos - b0) : p.list_rows[pos];
                                    buf[gq * p.capq + at + __popc(bal & lanemask_lt())] =
                                        make_uint2(__float_as_uint(group_key(p.metric, sums[st][qi])), id);
                                    if (at + __popc(bal) + kRound > p.capq) need = true;
                                }
                            }
                        }
                    }
                }
                // Counts only grow within a round, so the last appender to a
                // buffer sees its final count: the stamps of a round say
                // exactly "some buffer has less than a round of room left".
                if (need) s_need[g & 1u] = g;
                __syncwarp();
                if (lane == 0) mbar_arrive(rbar);
            }
        };
        if (p.metric == kMetricL2)
            scan_rounds(std::true_type{});
        else
            scan_rounds(std::false_type{});
        __syncthreads();
        if (tid == 0) fetch_item();  // overlaps the write-out below
        if (warp < ng) {
            uint32_t c = s_cnt[warp];
            uint2* bw = buf + warp * p.capq;
            if (c > p.r) {
                const uint32_t t = warp_select_compact(bw, c, p.r, hist + warp * 256u);
                if (lane == 0) atomicMin(&p.qbound[s_bound[G + warp]], t);
                c = p.r;
            } else if (c == p.r) {
                uint32_t t = 0;  // the R kept: their largest key bounds the query
                for (uint32_t i = lane; i < c; i += 32) t = max(t, ordered_key(__uint_as_float(bw[i].x)));
                t = __reduce_max_sync(0xffffffffu, t);
                if (lane == 0) atomicMin(&p.qbound[s_bound[G + warp]], t);
            }
            uint2* out = p.partial + static_cast<size_t>(p.pairs[first + warp]) * p.r;
            for (uint32_t i = lane; i < p.r; i += 32) out[i] = i < c ? bw[i] : make_uint2(0x7f800000u, 0xFFFFFFFFu);
        }
        __syncthreads();
    }
}

// One warp per query: exact distances of the R merged candidates, top-k by
// (distance, slot), written sorted. cand[q][r] = {approximate key, slot}
// (slot 0xFFFFFFFF = empty; any slot >= n is skipped the same way).
static __global__ void ivfpq_rerank_kernel(const float* __restrict__ queries, const float* __restrict__ vectors,
                                           const uint2* __restrict__ cand, uint32_t nq, uint32_t d, uint32_t r,
                                           uint32_t k, uint32_t rpow2, uint32_t n, int metric,
                                           float* __restrict__ out_dist, int64_t* __restrict__ out_rows) {
    extern __shared__ unsigned long long sbuf[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t warps = blockDim.x >> 5;
    const uint32_t q = blockIdx.x * warps + warp;
    if (q >= nq) return;
    unsigned long long* buf = sbuf + static_cast<size_t>(warp) * rpow2;
    const float* qv = queries + static_cast<size_t>(q) * d;
    for (uint32_t i = lane; i < rpow2; i += 32) {
        unsigned long long c = ~0ull;
        if (i < r) {
            const uint2 e = cand[static_cast<size_t>(q) * r + i];
            if (e.y < n) {  // 0xFFFFFFFF (none) and out-of-range slots are skipped
                const float* v = vectors + static_cast<size_t>(e.y) * d;
                float acc = 0.0f;
                if (metric == kMetricL2) {
                    for (uint32_t t = 0; t < d; ++t) {
                        const float df = __fsub_rn(qv[t], v[t]);
                        acc = __fadd_rn(acc, __fmul_rn(df, df));
                    }
                    acc = sqrtf(acc);
                } else {
                    for (uint32_t t = 0; t < d; ++t) acc = __fadd_rn(acc, __fmul_rn(qv[t], v[t]));
                    acc = finish_dot(metric, acc);
                }
                c = (static_cast<unsigned long long>(ordered_key(acc)) << 32) | e.y;
            }
        }
        buf[i] = c;
    }
    __syncwarp();
    for (uint32_t size = 2; size <= rpow2; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = lane; i < rpow2; i += 32) {
                const uint32_t j = i ^ stride;
                if (j > i) {
                    const unsigned long long a = buf[i], b = buf[j];
                    const bool up = (i & size) == 0;
                    if ((a > b) == up) {
                        buf[i] = b;
                        buf[j] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
    for (uint32_t i = lane; i < k; i += 32) {
        const unsigned long long c = i < rpow2 ? buf[i] : ~0ull;
        const bool valid = c != ~0ull;
        out_dist[static_cast<size_t>(q) * k + i] =
            valid ? key_to_float(static_cast<uint32_t>(c >> 32)) : __int_as_float(0x7f800000);
        out_rows[static_cast<size_t>(q) * k + i] = valid ? static_cast<int64_t>(c & 0xFFFFFFFFu) : -1;
    }
}

// Residuals x - centroid[list] in fp32, as GpuIVFPQIndex::rebuild_codes
// (GpuIVFPQIndex.cpp:105-113). One thread per element.
static __global__ void residuals_kernel(const float* __restrict__ vectors, const uint32_t* __restrict__ assign,
                                        const float* __restrict__ centroids, uint64_t n, uint32_t d,
                                        float* __restrict__ out) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n * d) return;
    const uint64_t r = t / d;
    const uint32_t i = static_cast<uint32_t>(t % d);
    out[t] = __fsub_rn(vectors[t], centroids[static_cast<size_t>(assign[r]) * d + i]);
}

// Gathers raw rows into list-major order: dst[pos] = src[rows[pos]] (d floats).
static __global__ void gather_rows_kernel(const float* __restrict__ src, const uint32_t* __restrict__ rows,
                                          uint64_t n, uint32_t d, float* __restrict__ dst) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n * d) return;
    const uint64_t pos = t / d;
    const uint32_t j = static_cast<uint32_t>(t % d);
    dst[t] = src[static_cast<size_t>(rows[pos]) * d + j];
}

// Gathers codes into list-major order: dst[pos] = src[rows[pos]].
static __global__ void gather_codes_kernel(const uint8_t* __restrict__ src, const uint32_t* __restrict__ rows,
                                           uint64_t n, uint32_t m, uint8_t* __restrict__ dst) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n * m) return;
    const uint64_t pos = t / m;
    const uint32_t j = static_cast<uint32_t>(t % m);
    dst[t] = src[static_cast<size_t>(rows[pos]) * m + j];
}

}  // namespace eb
