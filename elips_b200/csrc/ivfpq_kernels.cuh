// IVF-PQ search kernels, following GpuIVFPQIndex::search
// (src/gpu_engine/GpuIVFPQIndex.cpp:161-237):
//
//   1. probe: exact distances to every centroid + top-nprobe (the GpuPort
//      primitives in scan_kernels.cuh, as IvfIndexState::probe_lists,
//      src/gpu_engine/detail/IvfIndexState.cpp:395-423);
//   2. ivfpq_scan_kernel: one CTA per (query, probed list). The reference
//      decodes every candidate as centroid + codeword (fp32 add,
//      GpuIVFPQIndex.cpp:132-148) and takes elips::distance to it; here the
//      same per-dimension terms are tabulated once per (query, list) in a
//      lookup table [pq_dim][ksub] and summed per candidate. The terms are
//      identical, only the summation is grouped by subspace, so the
//      approximate ranking matches the reference's up to rounding; it only
//      decides which R = max(4k, k) candidates are reranked;
//   3. the k-best merge across probed lists (merge_topk_kernel);
//   4. ivfpq_rerank_kernel: exact elips::distance on the raw vectors of the R
//      candidates, sequential fp32 (exact_rank, :37-71), top-k by
//      (distance, slot).
#pragma once

#include <cstdint>

#include "scan_kernels.cuh"

namespace eb {

struct IvfPqParams {
    const float* queries;        // [nq][d]
    const float* centroids;      // [nlist][d]
    const float* codebook;       // [m][ksub][sub]
    const uint8_t* list_codes;   // [n][m], list-major (codes of list l at list_off[l])
    const uint32_t* list_rows;   // [n] slot of each list-major position
    const uint32_t* list_off;    // [nlist + 1]
    const uint32_t* probes;      // [nq][nprobe]
    uint2* partial;              // [nq][nprobe][r]
    uint32_t nq, d, nlist, nprobe, m, ksub, r, cap;
    int metric;
};

constexpr int kIvfThreads = 256;

// One CTA per (query, probe slot): blockIdx.x = q * nprobe + p.
static __global__ void __launch_bounds__(kIvfThreads) ivfpq_scan_kernel(const IvfPqParams p) {
    extern __shared__ uint8_t smem[];
    uint8_t* sp = smem;
    float* lut = reinterpret_cast<float*>(sp);
    sp += static_cast<size_t>(p.m) * p.ksub * sizeof(float);
    float* qv = reinterpret_cast<float*>(sp);
    sp += static_cast<size_t>(p.d) * sizeof(float);
    float* cv = reinterpret_cast<float*>(sp);
    sp += static_cast<size_t>(p.d) * sizeof(float);
    const BlockTopK st = btk_carve(sp, p.cap);

    const uint32_t q = blockIdx.x / p.nprobe, slot = blockIdx.x % p.nprobe;
    uint2* out = p.partial + static_cast<size_t>(blockIdx.x) * p.r;
    const uint32_t list = p.probes[static_cast<size_t>(q) * p.nprobe + slot];
    btk_init(st);
    if (list >= p.nlist) {  // fewer lists than nprobe: nothing to scan
        btk_finish(st, p.r, out);
        return;
    }
    for (uint32_t i = threadIdx.x; i < p.d; i += blockDim.x) {
        qv[i] = p.queries[static_cast<size_t>(q) * p.d + i];
        cv[i] = p.centroids[static_cast<size_t>(list) * p.d + i];
    }
    __syncthreads();
    const uint32_t sub = p.d / p.m;
    for (uint32_t e = threadIdx.x; e < p.m * p.ksub; e += blockDim.x) {
        const uint32_t mm = e / p.ksub, c = e % p.ksub;
        const float* cw = p.codebook + (static_cast<size_t>(mm) * p.ksub + c) * sub;
        float acc = 0.0f;
        for (uint32_t t = 0; t < sub; ++t) {
            const uint32_t dim = mm * sub + t;
            const float decoded = __fadd_rn(cv[dim], cw[t]);
            if (p.metric == kMetricL2) {
                const float df = __fsub_rn(qv[dim], decoded);
                acc = __fadd_rn(acc, __fmul_rn(df, df));
            } else {
                acc = __fadd_rn(acc, __fmul_rn(qv[dim], decoded));
            }
        }
        lut[e] = acc;
    }
    __syncthreads();
    const uint32_t b0 = p.list_off[list], b1 = p.list_off[list + 1];
    for (uint32_t base = b0; base < b1; base += blockDim.x) {
        const uint32_t j = base + threadIdx.x;
        const bool valid = j < b1;
        float key = 0.0f;
        uint32_t row = 0;
        if (valid) {
            const uint8_t* code = p.list_codes + static_cast<size_t>(j) * p.m;
            float sum = 0.0f;
            for (uint32_t mm = 0; mm < p.m; ++mm) sum = __fadd_rn(sum, lut[mm * p.ksub + code[mm]]);
            key = p.metric == kMetricL2 ? sqrtf(sum) : finish_dot(p.metric, sum);
            row = p.list_rows[j];
        }
        btk_offer(st, valid, key, row);
        btk_maybe_compact(st, p.r);
    }
    btk_finish(st, p.r, out);
}

// One warp per query: exact distances of the R merged candidates, top-k by
// (distance, slot), written sorted. cand[q][r] = {approximate key, slot}
// (slot 0xFFFFFFFF = empty).
static __global__ void ivfpq_rerank_kernel(const float* __restrict__ queries, const float* __restrict__ vectors,
                                           const uint2* __restrict__ cand, uint32_t nq, uint32_t d, uint32_t r,
                                           uint32_t k, uint32_t rpow2, int metric, float* __restrict__ out_dist,
                                           int64_t* __restrict__ out_rows) {
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
            if (e.y != 0xFFFFFFFFu) {
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
