// Index build on the device, bit-identical to the reference's trainers:
//
//   nearest_centroid_kernel  the assignment step of quant::detail::kmeans
//                            (src/quant_engine/KMeans.cpp:182-247, squared L2)
//                            and IvfIndexState::assign_vectors_to_centroids
//                            (src/gpu_engine/detail/IvfIndexState.cpp:167-191,
//                            elips::distance of the index metric)
//   centroid_update_kernel   the update step: member sums in ascending row
//                            order, mean by division (IVF) or by the
//                            reciprocal (quant), empty lists reseeded
//   centroid_normalize_kernel normalize_if_needed (IvfIndexState.cpp:20-35)
//
// Every distance is a strictly sequential single-precision chain with no
// fused multiply-add, as the reference's scalar loops (two chains per packed
// f32x2 instruction, each element rounded as the scalar one); the argmin keeps the
// lowest centroid among equal distances (strict '<' from FLT_MAX, centroid
// order ascending) and falls back to centroid 0 when no distance is below
// FLT_MAX (all NaN or infinite).
#pragma once

#include <cstdint>

#include "f32x2.cuh"

namespace eb {

enum : int { kTrainSqL2 = 0, kTrainL2 = 1, kTrainCos = 2, kTrainDot = 3 };

constexpr int kAsgRows = 64;    // rows per CTA (16 row groups of 4)
constexpr int kAsgCents = 64;   // centroids per tile (16 groups of 4)
constexpr int kAsgDims = 32;    // dimensions staged per step
constexpr int kAsgStride = 68;  // smem row pitch: float4-aligned, conflict-free transposed stores

__device__ __forceinline__ uint32_t train_ordered(float x) {
    const uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int MODE>
__device__ __forceinline__ float train_finish(float acc) {
    if (MODE == kTrainL2) return __fsqrt_rn(acc);
    if (MODE == kTrainCos) return __fsub_rn(1.0f, acc);
    if (MODE == kTrainDot) return -acc;
    return acc;
}

// Stages a [64 x w] block (row pitch ld, w <= 32) transposed into
// dst[dim][row]: lanes 8i..8i+7 read 8 consecutive dims of one row (32-byte
// sectors) and the transposed stores land on 32 distinct banks.
__device__ __forceinline__ void stage_tile(float* __restrict__ dst, const float* __restrict__ src, uint64_t ld,
                                           uint64_t first, uint64_t limit, uint32_t w) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t g = warp + 8u * i;
        const uint32_t rr = (g >> 2) * 4u + (lane >> 3);
        const uint32_t cc = (g & 3u) * 8u + (lane & 7u);
        const uint64_t r = first + rr;
        dst[cc * kAsgStride + rr] = (r < limit && cc < w) ? __ldg(src + r * ld + cc) : 0.0f;
    }
}

// keys[b * n + r] = b * key_stride + (nearest centroid of row r in batch b).
// Batch b reads columns [b * batch_cols, b * batch_cols + d) of every row and
// centroids cents[b][K][d]; a batch whose done flag is set is skipped. CTA:
// 256 threads = 16 x 16, each thread 4 rows x 4 centroids of every 64 x 64
// tile (16 sequential chains), dimensions staged 32 at a time.
template <int MODE>
__global__ void __launch_bounds__(256)
    nearest_centroid_kernel(const float* __restrict__ rows, uint64_t ld, uint64_t n, uint32_t d, uint32_t batch_cols,
                            const float* __restrict__ cents, uint32_t K, uint32_t key_stride,
                            uint32_t* __restrict__ keys, const uint32_t* __restrict__ done,
                            float* __restrict__ best_out) {
    __shared__ __align__(16) float rs[kAsgDims * kAsgStride];
    __shared__ __align__(16) float cs[kAsgDims * kAsgStride];
    const uint32_t b = blockIdx.y;
    if (done != nullptr && done[b] != 0u) return;
    rows += static_cast<uint64_t>(b) * batch_cols;
    cents += static_cast<uint64_t>(b) * K * d;
    const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * kAsgRows;
    const uint32_t ty = threadIdx.x >> 4, tx = threadIdx.x & 15u;
    float best[4];
    uint32_t arg[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        best[i] = 3.40282347e+38f;
        arg[i] = 0xFFFFFFFFu;
    }
    for (uint32_t c0 = 0; c0 < K; c0 += kAsgCents) {
        // acc2[i][h]: the chains of row i against centroids 2h and 2h + 1.
        unsigned long long acc2[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) acc2[i][0] = acc2[i][1] = 0ull;
        for (uint32_t k0 = 0; k0 < d; k0 += kAsgDims) {
            const uint32_t w = min(static_cast<uint32_t>(kAsgDims), d - k0);
            __syncthreads();
            stage_tile(rs, rows + k0, ld, r0, n, w);
            stage_tile(cs, cents + k0, d, c0, K, w);
            __syncthreads();
#pragma unroll 4
            for (uint32_t cc = 0; cc < w; ++cc) {
                const float4 a4 = *reinterpret_cast<const float4*>(rs + cc * kAsgStride + ty * 4u);
                const float4 c4 = *reinterpret_cast<const float4*>(cs + cc * kAsgStride + tx * 4u);
                const float av[4] = {a4.x, a4.y, a4.z, a4.w};
                const unsigned long long cp[2] = {f2_pack(c4.x, c4.y), f2_pack(c4.z, c4.w)};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const unsigned long long aa = f2_pack(av[i], av[i]);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (MODE == kTrainSqL2 || MODE == kTrainL2) {
                            const unsigned long long df = f2_sub(aa, cp[h]);
                            acc2[i][h] = f2_add(acc2[i][h], f2_prod(df, df));
                        } else {
                            acc2[i][h] = f2_add(acc2[i][h], f2_prod(aa, cp[h]));
                        }
                    }
                }
            }
        }
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f2_unpack(acc2[i][0], acc[i][0], acc[i][1]);
            f2_unpack(acc2[i][1], acc[i][2], acc[i][3]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t c = c0 + tx * 4u + j;
            if (c >= K) break;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float dist = train_finish<MODE>(acc[i][j]);
                if (dist < best[i]) {
                    best[i] = dist;
                    arg[i] = c;
                }
            }
        }
    }
    // Each thread's centroids ascend, so its winner is the lowest index among
    // its equal minima; across the 16 threads of a row the (distance, index)
    // minimum keeps that rule (-0 and +0 compare equal, as '<' does).
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        unsigned long long key = arg[i] == 0xFFFFFFFFu
                                     ? ~0ull
                                     : (static_cast<unsigned long long>(train_ordered(__fadd_rn(best[i], 0.0f))) << 32) |
                                           arg[i];
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, key, off);
            key = o < key ? o : key;
        }
        const uint64_t r = r0 + ty * 4u + i;
        if (tx == 0 && r < n)
            keys[static_cast<uint64_t>(b) * n + r] =
                b * key_stride + (key == ~0ull ? 0u : static_cast<uint32_t>(key & 0xFFFFFFFFull));
        // The winner's distance (optional), written by the thread that owns
        // the winning centroid (its own bits: -0 stays -0); FLT_MAX when no
        // distance was below it, the reference's best_distance in that case.
        if (best_out != nullptr && r < n) {
            if (key == ~0ull) {
                if (tx == 0) best_out[static_cast<uint64_t>(b) * n + r] = 3.40282347e+38f;
            } else if (arg[i] == static_cast<uint32_t>(key & 0xFFFFFFFFull)) {
                best_out[static_cast<uint64_t>(b) * n + r] = best[i];
            }
        }
    }
}

// vals[b * n + r] = r.
static __global__ void row_iota_kernel(uint32_t* __restrict__ vals, uint64_t n, uint64_t total) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t < total) vals[t] = static_cast<uint32_t>(t % n);
}

// [start, end) of every key in the sorted key array (untouched for absent keys).
static __global__ void segment_bounds_kernel(const uint32_t* __restrict__ keys, uint64_t total,
                                             uint32_t* __restrict__ start, uint32_t* __restrict__ end) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const uint32_t k = keys[t];
    if (t == 0 || keys[t - 1] != k) start[k] = static_cast<uint32_t>(t);
    if (t + 1 == total || keys[t + 1] != k) end[k] = static_cast<uint32_t>(t + 1);
}

// cents[b][c][i] = row (min(n-1, c * stride)) of batch b.
static __global__ void seed_centroids_kernel(const float* __restrict__ rows, uint64_t ld, uint64_t n, uint32_t d,
                                             uint32_t batch_cols, uint32_t K, uint64_t total, uint64_t stride,
                                             float* __restrict__ cents) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const uint32_t i = static_cast<uint32_t>(t % d);
    const uint64_t c = (t / d) % K, b = t / (static_cast<uint64_t>(d) * K);
    uint64_t sample = c * stride;
    if (sample > n - 1) sample = n - 1;
    cents[t] = rows[b * batch_cols + sample * ld + i];
}

// One thread per (batch, centroid, dimension): the sum of the members'
// values in ascending row order (members = rows sorted stably by key), then
//   IVF   (IvfIndexState.cpp:148-158): sum / float(count); empty -> row
//         min(n-1, c % n)
//   quant (KMeans.cpp:222-241): sum * (1 / float(count)); empty -> row c % n;
//         moved[b] set when any value changes or a centroid is reseeded.
template <bool IVF>
__global__ void __launch_bounds__(256)
    centroid_update_kernel(const float* __restrict__ rows, uint64_t ld, uint64_t n, uint32_t d, uint32_t batch_cols,
                           const uint32_t* __restrict__ members, const uint32_t* __restrict__ start,
                           const uint32_t* __restrict__ end, uint32_t K, uint64_t total, float* __restrict__ cents,
                           uint32_t* __restrict__ moved, const uint32_t* __restrict__ done) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const uint32_t i = static_cast<uint32_t>(t % d);
    const uint64_t key = t / d;
    const uint32_t b = static_cast<uint32_t>(key / K);
    const uint32_t c = static_cast<uint32_t>(key % K);
    if (done != nullptr && done[b] != 0u) return;
    const float* col = rows + static_cast<uint64_t>(b) * batch_cols + i;
    const uint32_t s = start[key], e = end[key];
    if (e <= s) {
        cents[t] = col[(c % n) * ld];
        if (!IVF) moved[b] = 1u;
        return;
    }
    float sum = 0.0f;
    uint32_t j = s;
    for (; j + 8 <= e; j += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldg(col + static_cast<uint64_t>(__ldg(members + j + u)) * ld);
#pragma unroll
        for (int u = 0; u < 8; ++u) sum = __fadd_rn(sum, v[u]);
    }
    for (; j < e; ++j) sum = __fadd_rn(sum, __ldg(col + static_cast<uint64_t>(__ldg(members + j)) * ld));
    const float count = __uint2float_rn(e - s);
    if (IVF) {
        cents[t] = __fdiv_rn(sum, count);
    } else {
        const float upd = __fmul_rn(sum, __fdiv_rn(1.0f, count));
        if (upd != cents[t]) moved[b] = 1u;
        cents[t] = upd;
    }
}

// normalize_if_needed for the cosine metric: norm = sqrt of the sequential
// sum of squares; a centroid whose norm is <= 0 stays as it is.
static __global__ void centroid_normalize_kernel(float* __restrict__ cents, uint32_t K, uint32_t d) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= K) return;
    float* v = cents + static_cast<uint64_t>(c) * d;
    float sum = 0.0f;
    for (uint32_t i = 0; i < d; ++i) sum = __fadd_rn(sum, __fmul_rn(v[i], v[i]));
    const float norm = __fsqrt_rn(sum);
    if (norm <= 0.0f) return;
    for (uint32_t i = 0; i < d; ++i) v[i] = __fdiv_rn(v[i], norm);
}

// codes[r * m + s] = keys[s * n + r] (the [subspace][row] argmin output
// turned into row-major PQ codes).
static __global__ void keys_to_codes_kernel(const uint32_t* __restrict__ keys, uint64_t n, uint32_t m,
                                            uint8_t* __restrict__ codes) {
    const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n * m) return;
    const uint64_t r = t / m;
    const uint32_t s = static_cast<uint32_t>(t % m);
    codes[t] = static_cast<uint8_t>(keys[static_cast<uint64_t>(s) * n + r]);
}

// done[b] |= !moved[b]; moved[b] = 0 (the early stop of KMeans.cpp:243-245).
static __global__ void kmeans_flags_kernel(uint32_t* __restrict__ moved, uint32_t* __restrict__ done, uint32_t batch) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= batch) return;
    if (moved[b] == 0u) done[b] = 1u;
    moved[b] = 0u;
}

}  // namespace eb
