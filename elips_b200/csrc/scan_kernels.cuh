// SIMT kernels that reproduce the reference's scalar arithmetic bit for bit:
// strictly sequential single-precision sums with no fused multiply-add
// (explicit __fadd_rn / __fmul_rn / __fsub_rn), IEEE square root.
//
//   distances_kernel     GpuPort::compute_distances_batch (GpuPort.hpp:65-73)
//                        with elips::distance (src/Metrics.cpp:20-37,104-115)
//   topk_rows_kernel     GpuPort::top_k (GpuPort.hpp:75-82)
//   pq_lut / pq_scan     ProductQuantizer::make_lut + lut_distance
//                        (src/quant_engine/ProductQuantizer.cpp:118-183)
//   sq8_lut / sq8_scan   ScalarQuantizer::make_lut + lut_distance
//                        (src/quant_engine/ScalarQuantizer.cpp:83-128)
//   sq8_encode           ScalarQuantizer::encode (ScalarQuantizer.cpp:52-68)
//   rotate_rows          detail::apply_matrix for OPQ (KMeans.cpp:295-305)
#pragma once

#include <cstdint>

#include "block_select.cuh"
#include "f32x2.cuh"

namespace eb {

enum : int { kMetricCos = 0, kMetricL2 = 1, kMetricDot = 2 };

// Post-processing of a sequential sum, as the reference's distance / lut_distance.
__device__ __forceinline__ float finish_dot(int metric, float dot) {
    if (metric == kMetricCos) return __fsub_rn(1.0f, dot);
    return -dot;
}

// ------------------------------------------------------------- distances

constexpr int kDistRows = 128;   // database rows per CTA (one per thread)
constexpr int kDistQ = 8;        // queries per CTA
constexpr int kDistDims = 32;    // dimensions staged per step

// out[q * nb + r] = elips::distance(metric, queries[q], db[r]) exactly. A
// thread owns one base row and 8 queries: 8 sequential chains, advanced in
// pairs by packed f32x2 operations (each element rounded as the scalar .rn
// operation); the 8 query values of a dimension are read as two float4.
template <bool L2>
__device__ __forceinline__ void distance_chains(const float (*dbs)[kDistDims + 1], const float (*qst)[kDistQ],
                                                uint32_t t, uint32_t w, unsigned long long (&acc)[kDistQ / 2]) {
    for (uint32_t c = 0; c < w; ++c) {
        const float b = dbs[t][c];
        const unsigned long long bb = f2_pack(b, b);
        const float4 qa = *reinterpret_cast<const float4*>(&qst[c][0]);
        const float4 qb = *reinterpret_cast<const float4*>(&qst[c][4]);
        const unsigned long long qp[kDistQ / 2] = {f2_pack(qa.x, qa.y), f2_pack(qa.z, qa.w), f2_pack(qb.x, qb.y),
                                                   f2_pack(qb.z, qb.w)};
#pragma unroll
        for (int j = 0; j < kDistQ / 2; ++j) {
            if (L2) {
                const unsigned long long df = f2_sub(qp[j], bb);
                acc[j] = f2_add(acc[j], f2_prod(df, df));
            } else {
                acc[j] = f2_add(acc[j], f2_prod(qp[j], bb));
            }
        }
    }
}

static __global__ void __launch_bounds__(kDistRows)
    distances_kernel(const float* __restrict__ queries, const float* __restrict__ db, uint32_t nq,
                     uint32_t nb, uint32_t d, int metric, float* __restrict__ out) {
    static_assert(kDistQ == 8, "two float4 of queries per dimension");
    __shared__ float dbs[kDistRows][kDistDims + 1];
    __shared__ __align__(16) float qst[kDistDims][kDistQ];
    const uint32_t r0 = blockIdx.x * kDistRows, q0 = blockIdx.y * kDistQ;
    const uint32_t t = threadIdx.x;
    unsigned long long acc[kDistQ / 2];
#pragma unroll
    for (int j = 0; j < kDistQ / 2; ++j) acc[j] = 0ull;
    for (uint32_t base = 0; base < d; base += kDistDims) {
        const uint32_t w = min(static_cast<uint32_t>(kDistDims), d - base);
        __syncthreads();
        for (uint32_t i = t; i < kDistRows * kDistDims; i += kDistRows) {
            const uint32_t rr = i / kDistDims, c = i % kDistDims;
            const uint32_t r = r0 + rr;
            dbs[rr][c] = (r < nb && c < w) ? db[static_cast<size_t>(r) * d + base + c] : 0.0f;
        }
        for (uint32_t i = t; i < kDistQ * kDistDims; i += kDistRows) {
            const uint32_t qq = i / kDistDims, c = i % kDistDims;
            const uint32_t q = q0 + qq;
            qst[c][qq] = (q < nq && c < w) ? queries[static_cast<size_t>(q) * d + base + c] : 0.0f;
        }
        __syncthreads();
        if (metric == kMetricL2) distance_chains<true>(dbs, qst, t, w, acc);
        else distance_chains<false>(dbs, qst, t, w, acc);
    }
    const uint32_t r = r0 + t;
    if (r >= nb) return;
    float accs[kDistQ];
#pragma unroll
    for (int j = 0; j < kDistQ / 2; ++j) f2_unpack(acc[j], accs[2 * j], accs[2 * j + 1]);
#pragma unroll
    for (int j = 0; j < kDistQ; ++j) {
        const uint32_t q = q0 + j;
        if (q >= nq) break;
        out[static_cast<size_t>(q) * nb + r] = metric == kMetricL2 ? sqrtf(accs[j]) : finish_dot(metric, accs[j]);
    }
}

// --------------------------------------------------------- normalisation

constexpr int kNormRows = 32;  // rows per CTA (one per thread of warp 0)
constexpr int kNormDims = 32;  // dimensions staged per step

// out = Vector::normalized (include/elips/domain/Vector.hpp:25-44) of every
// row: magnitude = sqrt of the sequential sum of v*v (no FMA), each value
// divided by it (IEEE), zero rows copied unchanged. A CTA stages 32 rows x 32
// dimensions at a time (coalesced) so each of its first 32 threads can sum
// its row in order; all threads then write the quotients.
static __global__ void __launch_bounds__(256)
    normalize_rows_kernel(const float* __restrict__ in, float* __restrict__ out, uint64_t n, uint32_t d) {
    __shared__ float tile[kNormRows][kNormDims + 1];
    __shared__ float mag[kNormRows];
    const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * kNormRows;
    const uint32_t tid = threadIdx.x;
    float sum = 0.0f;
    for (uint32_t c0 = 0; c0 < d; c0 += kNormDims) {
        for (uint32_t e = tid; e < kNormRows * kNormDims; e += blockDim.x) {
            const uint32_t rr = e / kNormDims, cc = e % kNormDims;
            const uint64_t row = r0 + rr;
            tile[rr][cc] = (row < n && c0 + cc < d) ? in[row * d + c0 + cc] : 0.0f;
        }
        __syncthreads();
        if (tid < kNormRows) {
            const uint32_t lim = min(static_cast<uint32_t>(kNormDims), d - c0);
            for (uint32_t cc = 0; cc < lim; ++cc) sum = __fadd_rn(sum, __fmul_rn(tile[tid][cc], tile[tid][cc]));
        }
        __syncthreads();
    }
    if (tid < kNormRows) mag[tid] = sqrtf(sum);
    __syncthreads();
    const uint64_t left = n > r0 ? n - r0 : 0ull;
    const uint64_t rows = left < static_cast<uint64_t>(kNormRows) ? left : static_cast<uint64_t>(kNormRows);
    for (uint64_t e = tid; e < rows * d; e += blockDim.x) {
        const uint32_t rr = static_cast<uint32_t>(e / d);
        const float m = mag[rr];
        const float x = in[r0 * d + e];
        out[r0 * d + e] = m == 0.0f ? x : __fdiv_rn(x, m);
    }
}

// ------------------------------------------------------------ block sort

// Ascending bitonic sort of n (power of two) composites in shared memory.
__device__ __forceinline__ void block_bitonic_sort(unsigned long long* a, uint32_t n) {
    for (uint32_t size = 2; size <= n; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
                const uint32_t j = i ^ stride;
                if (j > i) {
                    const unsigned long long x = a[i], y = a[j];
                    const bool up = (i & size) == 0;
                    if ((x > y) == up) {
                        a[i] = y;
                        a[j] = x;
                    }
                }
            }
        }
    }
    __syncthreads();
}

// Shared-memory carve-out for one BlockTopK of capacity cap.
__device__ __forceinline__ BlockTopK btk_carve(uint8_t*& p, uint32_t cap) {
    BlockTopK s;
    s.buf = reinterpret_cast<uint2*>(p);
    p += cap * sizeof(uint2);
    s.tmp = reinterpret_cast<uint2*>(p);
    p += cap * sizeof(uint2);
    s.hist = reinterpret_cast<uint32_t*>(p);
    p += 256 * sizeof(uint32_t);
    s.cnt = reinterpret_cast<uint32_t*>(p);
    s.thr = reinterpret_cast<float*>(p + 4);
    s.sel = reinterpret_cast<uint32_t*>(p + 8);
    p += 32;
    s.cap = cap;
    return s;
}

__host__ __device__ constexpr uint32_t btk_bytes(uint32_t cap) { return cap * 16u + 1024u + 32u; }

// ---------------------------------------------------------- GpuPort::top_k

// One CTA per query row: the k smallest (value, index) of dist[q][0..nb),
// ascending, ties by index. indices_out / values_out are [nq][k].
static __global__ void topk_rows_kernel(const float* __restrict__ dist, uint32_t nq, uint32_t nb, uint32_t k,
                                 uint32_t cap, uint32_t kpow2, uint32_t* __restrict__ idx_out,
                                 float* __restrict__ val_out) {
    extern __shared__ uint8_t smem[];
    uint8_t* p = smem;
    const BlockTopK s = btk_carve(p, cap);
    unsigned long long* sorted = reinterpret_cast<unsigned long long*>(p);
    const uint32_t q = blockIdx.x;
    if (q >= nq) return;
    btk_init(s);
    const float* row = dist + static_cast<size_t>(q) * nb;
    for (uint32_t base = 0; base < nb; base += blockDim.x) {
        const uint32_t i = base + threadIdx.x;
        btk_offer(s, i < nb, i < nb ? row[i] : 0.0f, i);
        btk_maybe_compact(s, k);
    }
    btk_compact(s, k);
    const uint32_t c = *s.cnt;
    for (uint32_t j = threadIdx.x; j < kpow2; j += blockDim.x) sorted[j] = j < c ? composite_of(s.buf[j]) : ~0ull;
    block_bitonic_sort(sorted, kpow2);
    for (uint32_t j = threadIdx.x; j < k; j += blockDim.x) {
        const unsigned long long e = sorted[j];
        const bool valid = j < c;
        idx_out[static_cast<size_t>(q) * k + j] = valid ? static_cast<uint32_t>(e & 0xFFFFFFFFu) : 0xFFFFFFFFu;
        val_out[static_cast<size_t>(q) * k + j] =
            valid ? key_to_float(static_cast<uint32_t>(e >> 32)) : __int_as_float(0x7f800000);
    }
}

// -------------------------------------------------------------- OPQ rotate

// out[r] = R x in[r] with apply_matrix's order: out_i = sum_j R[i][j] * v[j],
// sequential over j (KMeans.cpp:295-305). One thread per (row, i).
static __global__ void rotate_rows_kernel(const float* __restrict__ rot, const float* __restrict__ in, uint64_t rows,
                                   uint32_t d, float* __restrict__ out) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= rows * d) return;
    const uint64_t r = t / d;
    const uint32_t i = static_cast<uint32_t>(t % d);
    const float* v = in + r * d;
    const float* m = rot + static_cast<size_t>(i) * d;
    float sum = 0.0f;
    for (uint32_t j = 0; j < d; ++j) sum = __fadd_rn(sum, __fmul_rn(m[j], v[j]));
    out[t] = sum;
}

// ------------------------------------------------------------------- PQ

// lut[q][m][c] per ProductQuantizer::make_lut: -sum q_s*c (cos, dot) or
// sum (q_s - c)^2 (euclidean), sequential over sub_dim. One thread per entry.
static __global__ void pq_lut_kernel(const float* __restrict__ queries, const float* __restrict__ codebook,
                              uint32_t nq, uint32_t d, uint32_t m_sub, uint32_t ksub, int metric,
                              float* __restrict__ lut) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t per_q = static_cast<uint64_t>(m_sub) * ksub;
    if (t >= nq * per_q) return;
    const uint32_t q = static_cast<uint32_t>(t / per_q);
    const uint32_t rem = static_cast<uint32_t>(t % per_q);
    const uint32_t m = rem / ksub, c = rem % ksub;
    const uint32_t sub = d / m_sub;
    const float* qs = queries + static_cast<size_t>(q) * d + static_cast<size_t>(m) * sub;
    const float* cen = codebook + (static_cast<size_t>(m) * ksub + c) * sub;
    float acc = 0.0f;
    if (metric == kMetricL2) {
        for (uint32_t i = 0; i < sub; ++i) {
            const float df = __fsub_rn(qs[i], cen[i]);
            acc = __fadd_rn(acc, __fmul_rn(df, df));
        }
        lut[t] = acc;
    } else {
        for (uint32_t i = 0; i < sub; ++i) acc = __fadd_rn(acc, __fmul_rn(qs[i], cen[i]));
        lut[t] = -acc;
    }
}

// lut_distance post-processing (ProductQuantizer.cpp:170-181,
// ScalarQuantizer.cpp:119-126).
__device__ __forceinline__ float lut_finish(int metric, float sum) {
    if (metric == kMetricCos) return __fadd_rn(1.0f, sum);
    if (metric == kMetricDot) return sum;
    return sqrtf(fmaxf(0.0f, sum));
}

constexpr int kScanThreads = 256;
constexpr int kPqQueriesPerCta = 4;

// Exhaustive PQ ADC scan. grid = (splits, ceil(nq / 4)); CTA: 4 queries' LUTs
// in shared memory, rows [split range) in rounds of 256 (one row per thread),
// sum over m sequential, one running top-k per query; writes
// partial[q][split][k].
static __global__ void __launch_bounds__(kScanThreads)
    pq_scan_kernel(const float* __restrict__ lut, const uint8_t* __restrict__ codes, uint32_t n, uint32_t nq,
                   uint32_t m_sub, uint32_t ksub, int metric, uint32_t k, uint32_t cap, uint32_t splits,
                   uint2* __restrict__ partial) {
    extern __shared__ uint8_t smem[];
    uint8_t* p = smem;
    const uint32_t lut_floats = m_sub * ksub;
    float* luts = reinterpret_cast<float*>(p);
    p += kPqQueriesPerCta * lut_floats * sizeof(float);
    BlockTopK st[kPqQueriesPerCta];
#pragma unroll
    for (int j = 0; j < kPqQueriesPerCta; ++j) st[j] = btk_carve(p, cap);
    const uint32_t q0 = blockIdx.y * kPqQueriesPerCta;
    const uint32_t sp = blockIdx.x;
    for (uint32_t i = threadIdx.x; i < kPqQueriesPerCta * lut_floats; i += blockDim.x) {
        const uint32_t j = i / lut_floats;
        luts[i] = (q0 + j < nq) ? lut[static_cast<size_t>(q0 + j) * lut_floats + (i % lut_floats)] : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kPqQueriesPerCta; ++j) btk_init(st[j]);
    const uint32_t r0 = static_cast<uint32_t>(static_cast<uint64_t>(sp) * n / splits);
    const uint32_t r1 = static_cast<uint32_t>(static_cast<uint64_t>(sp + 1) * n / splits);
    for (uint32_t base = r0; base < r1; base += blockDim.x) {
        const uint32_t r = base + threadIdx.x;
        const bool valid = r < r1;
        float sum[kPqQueriesPerCta];
#pragma unroll
        for (int j = 0; j < kPqQueriesPerCta; ++j) sum[j] = 0.0f;
        if (valid) {
            const uint8_t* code = codes + static_cast<size_t>(r) * m_sub;
            for (uint32_t m = 0; m < m_sub; ++m) {
                const uint32_t c = code[m];
#pragma unroll
                for (int j = 0; j < kPqQueriesPerCta; ++j)
                    sum[j] = __fadd_rn(sum[j], luts[j * lut_floats + m * ksub + c]);
            }
        }
#pragma unroll
        for (int j = 0; j < kPqQueriesPerCta; ++j) {
            btk_offer(st[j], valid && q0 + j < nq, lut_finish(metric, sum[j]), r);
            btk_maybe_compact(st[j], k);
        }
    }
#pragma unroll
    for (int j = 0; j < kPqQueriesPerCta; ++j) {
        const uint32_t q = q0 + j;
        if (q < nq) btk_finish(st[j], k, partial + (static_cast<size_t>(q) * splits + sp) * k);
    }
}

// ------------------------------------------------------------------- SQ8

// lut[q][i][level] per ScalarQuantizer::make_lut: value = min + level*scale;
// -(q*value) (cos, dot) or (q - value)^2 (euclidean).
static __global__ void sq8_lut_kernel(const float* __restrict__ queries, const float* __restrict__ mins,
                               const float* __restrict__ scales, uint32_t nq, uint32_t d, int metric,
                               float* __restrict__ lut) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t per_q = static_cast<uint64_t>(d) * 256u;
    if (t >= nq * per_q) return;
    const uint32_t q = static_cast<uint32_t>(t / per_q);
    const uint32_t rem = static_cast<uint32_t>(t % per_q);
    const uint32_t i = rem >> 8, level = rem & 255u;
    const float value = __fadd_rn(mins[i], __fmul_rn(static_cast<float>(level), scales[i]));
    const float qv = queries[static_cast<size_t>(q) * d + i];
    if (metric == kMetricL2) {
        const float df = __fsub_rn(qv, value);
        lut[t] = __fmul_rn(df, df);
    } else {
        lut[t] = -__fmul_rn(qv, value);
    }
}

// Exhaustive sq8 ADC scan, one query per CTA: grid = (splits, nq). The
// query's d x 256 LUT is staged in shared memory when lut_in_smem (d <= 192),
// else read from global memory. Sum over the d dimensions is sequential.
static __global__ void __launch_bounds__(kScanThreads)
    sq8_scan_kernel(const float* __restrict__ lut, const uint8_t* __restrict__ codes, uint32_t n, uint32_t d,
                    int metric, uint32_t k, uint32_t cap, uint32_t splits, int lut_in_smem,
                    uint2* __restrict__ partial) {
    extern __shared__ uint8_t smem[];
    uint8_t* p = smem;
    const BlockTopK st = btk_carve(p, cap);
    float* slut = reinterpret_cast<float*>(p);
    const uint32_t q = blockIdx.y, sp = blockIdx.x;
    const float* qlut = lut + static_cast<size_t>(q) * d * 256u;
    if (lut_in_smem) {
        for (uint32_t i = threadIdx.x; i < d * 256u; i += blockDim.x) slut[i] = qlut[i];
        qlut = slut;
    }
    btk_init(st);
    const uint32_t r0 = static_cast<uint32_t>(static_cast<uint64_t>(sp) * n / splits);
    const uint32_t r1 = static_cast<uint32_t>(static_cast<uint64_t>(sp + 1) * n / splits);
    for (uint32_t base = r0; base < r1; base += blockDim.x) {
        const uint32_t r = base + threadIdx.x;
        const bool valid = r < r1;
        float sum = 0.0f;
        if (valid) {
            const uint8_t* code = codes + static_cast<size_t>(r) * d;
            for (uint32_t i = 0; i < d; ++i) sum = __fadd_rn(sum, qlut[i * 256u + code[i]]);
        }
        btk_offer(st, valid, lut_finish(metric, sum), r);
        btk_maybe_compact(st, k);
    }
    btk_finish(st, k, partial + (static_cast<size_t>(q) * splits + sp) * k);
}

// ScalarQuantizer::encode: level = (x - min) / scale, clamp to [0, 255],
// round half away from zero. One thread per element.
static __global__ void sq8_encode_kernel(const float* __restrict__ rows, const float* __restrict__ mins,
                                  const float* __restrict__ scales, uint64_t n, uint32_t d,
                                  uint8_t* __restrict__ codes) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n * d) return;
    const uint32_t i = static_cast<uint32_t>(t % d);
    const float level = __fdiv_rn(__fsub_rn(rows[t], mins[i]), scales[i]);
    const float clamped = fminf(fmaxf(level, 0.0f), 255.0f);
    codes[t] = static_cast<uint8_t>(lroundf(clamped));
}

}  // namespace eb
