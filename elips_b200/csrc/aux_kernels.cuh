// Operand preparation and final top-k merge kernels for the exact search.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace eb {

// Rounds fp32 to tf32 (round to nearest, ties away) in an fp32 container.
__device__ __forceinline__ float to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// One warp per row: converts fp32 rows [rows x d] to the tensor-core operand
// layout [rows x d_pad] (zero padded to a whole number of 128-byte K blocks)
// and writes the squared norm of the stored (rounded) row when norms != null.
//   kind 0: fp16, 1: bf16, 2: tf32 split (hi to out, x - hi to out_lo).
__global__ void prep_rows_f32_kernel(const float* __restrict__ in, uint64_t rows, uint32_t d,
                                     uint32_t d_pad, int kind, void* __restrict__ out,
                                     float* __restrict__ out_lo, float* __restrict__ norms) {
    const uint64_t row = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    if (row >= rows) return;
    const float* src = in + row * d;
    float acc = 0.0f;
    for (uint32_t j = lane; j < d_pad; j += 32) {
        const float x = j < d ? src[j] : 0.0f;
        float stored;
        if (kind == 0) {
            const __half h = __float2half_rn(x);
            reinterpret_cast<__half*>(out)[row * d_pad + j] = h;
            stored = __half2float(h);
        } else if (kind == 1) {
            const __nv_bfloat16 h = __float2bfloat16_rn(x);
            reinterpret_cast<__nv_bfloat16*>(out)[row * d_pad + j] = h;
            stored = __bfloat162float(h);
        } else {
            const float hi = to_tf32(x);
            reinterpret_cast<float*>(out)[row * d_pad + j] = hi;
            out_lo[row * d_pad + j] = x - hi;
            stored = x;
        }
        acc = fmaf(stored, stored, acc);
    }
    if (norms != nullptr) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) norms[row] = acc;
    }
}

// int8 rows [rows x d] -> [rows x d_pad], zero padded.
__global__ void prep_rows_i8_kernel(const int8_t* __restrict__ in, uint64_t rows, uint32_t d,
                                    uint32_t d_pad, int8_t* __restrict__ out) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * d_pad) return;
    const uint64_t r = i / d_pad;
    const uint32_t j = static_cast<uint32_t>(i % d_pad);
    out[i] = j < d ? in[r * d + j] : int8_t(0);
}

// Radix select, 8 bits per pass, over n composites read by get(j): finds
// the group of the rank-th smallest (1-based) among those whose bits under
// `pmask` equal `prefix` (pass the common high bits in, zero for none).
// Passes start at byte `first` (0 = the top byte); selection stops as soon as
// the chosen bin holds exactly the remaining rank, so on return the selected
// elements are: every composite with (c & pmask) < prefix, and of those with
// (c & pmask) == prefix, `rank` in any order (all of them when it stopped
// early; copies of one value otherwise). One warp; hist = its 256 words.
template <class Get>
__device__ __forceinline__ void warp_radix_select(Get get, uint32_t n, uint32_t& rank, unsigned long long& prefix,
                                                  unsigned long long& pmask, int first, uint32_t* hist) {
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll 1
    for (int pass = first; pass < 8; ++pass) {
        const uint32_t shift = 56u - 8u * static_cast<uint32_t>(pass);
        for (uint32_t b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
        for (uint32_t j0 = 0; j0 < n; j0 += 128) {
            unsigned long long c[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t j = j0 + u * 32 + lane;
                c[u] = j < n ? get(j) : 0ull;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t j = j0 + u * 32 + lane;
                if (j < n && (c[u] & pmask) == prefix) atomicAdd(&hist[(c[u] >> shift) & 255u], 1u);
            }
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
        uint32_t digit = 0, before = excl, inbin = 0;
        if (mine) {
            uint32_t acc = excl;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (acc + bins[i] >= rank) {
                    digit = lane * 8 + i;
                    before = acc;
                    inbin = bins[i];
                    break;
                }
                acc += bins[i];
            }
        }
        const uint32_t owner = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
        digit = __shfl_sync(0xffffffffu, digit, owner);
        before = __shfl_sync(0xffffffffu, before, owner);
        inbin = __shfl_sync(0xffffffffu, inbin, owner);
        rank -= before;
        prefix |= static_cast<unsigned long long>(digit) << shift;
        pmask |= 255ull << shift;
        __syncwarp();
        if (inbin == rank) break;  // the whole bin is selected
    }
}

// Ascending bitonic sort of n (power of two) composites by one warp.
__device__ __forceinline__ void warp_bitonic_sort(unsigned long long* buf, uint32_t n) {
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t size = 2; size <= n; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = lane; i < n; i += 32) {
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
}

// One warp selects the `take` smallest of `count` composites read by get(j)
// into buf[0, w) (unsorted); returns w (= take when at least take are real,
// padding {+inf, 0xFFFFFFFF} included only to fill up otherwise). A first
// pass finds the leading bits shared by all real candidates (the keys of one
// query's candidates are close, so the top byte or two agree), the radix
// select starts below them and stops once a bin is taken whole; the
// survivors are then gathered.
template <class Get>
__device__ __forceinline__ uint32_t merge_select(Get get, uint32_t count, uint32_t take, uint32_t* hist,
                                                 unsigned long long* buf) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t lt = lanemask_lt();
    uint32_t w = 0;
    // the real candidates: how many, and the high bits they all share
    uint32_t real = 0;
    unsigned long long first_c = 0, diff = 0;
    bool have = false;
    for (uint32_t j0 = 0; j0 < count; j0 += 128) {
        unsigned long long c[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t j = j0 + u * 32 + lane;
            c[u] = j < count ? get(j) : ~0ull;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const bool is_real = (c[u] & 0xFFFFFFFFull) != 0xFFFFFFFFull;
            const uint32_t m = __ballot_sync(0xffffffffu, is_real);
            real += __popc(m);
            if (m != 0 && !have) {
                first_c = __shfl_sync(0xffffffffu, c[u], __ffs(m) - 1);
                have = true;
            }
            if (is_real) diff |= c[u] ^ first_c;
        }
    }
    unsigned long long prefix = 0, pmask = 0;
    uint32_t rank = take;
    int first = 0;
    if (real >= take) {
        // select among the real ones only: start below their common bits
        diff = __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(diff >> 32)) * (1ull << 32) |
               __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(diff));
        const int top = diff == 0 ? 0 : 63 - __clzll(static_cast<long long>(diff));
        first = (63 - top) / 8;
        pmask = first == 0 ? 0ull : ~0ull << (64 - 8 * first);
        prefix = first_c & pmask;
    }
    warp_radix_select(get, count, rank, prefix, pmask, first, hist);
    // every composite below the selected group, then `rank` of the group
    for (uint32_t j0 = 0; j0 < count; j0 += 32) {
        const uint32_t j = j0 + lane;
        const unsigned long long c = j < count ? get(j) : ~0ull;
        const bool keep = j < count && (c & pmask) < prefix &&
                          (real < take || (c & 0xFFFFFFFFull) != 0xFFFFFFFFull);
        const uint32_t m = __ballot_sync(0xffffffffu, keep);
        if (keep) buf[w + __popc(m & lt)] = c;
        w += __popc(m);
    }
    const uint32_t target = w + rank;
    for (uint32_t j0 = 0; j0 < count && w < target; j0 += 32) {
        const uint32_t j = j0 + lane;
        const unsigned long long c = j < count ? get(j) : ~0ull;
        const bool eq = j < count && (c & pmask) == prefix;
        const uint32_t m = __ballot_sync(0xffffffffu, eq);
        const uint32_t pos = w + __popc(m & lt);
        if (eq && pos < target) buf[pos] = c;
        w = min(target, w + __popc(m));
    }
    return w;
}

__device__ __forceinline__ unsigned long long merge_composite(uint2 e) {
    return (static_cast<unsigned long long>(ordered_key(__uint_as_float(e.x))) << 32) | e.y;
}

// Final top-k per query: one warp selects the k smallest (key, row) pairs
// among `lists` candidate lists of `len` (>= k) entries each and writes
// them sorted.
// List l of query q starts at cand + q*stride_q + l*stride_l (entries).
// With sub > 1 each query's lists are cut into `sub` groups of `lists` lists
// (the last group: `lists_last`), one warp per (query, group), and output row
// q*sub + j holds group j's k best: the first stage of a two-stage merge.
// Composite 64-bit keys (ordered key << 32 | row) are unique except the
// padding {+inf, 0xFFFFFFFF}. When a query has at most `cache_cap`
// candidates they are read from global memory once (16-byte loads where the
// lists are contiguous and aligned) into the warp's shared-memory cache,
// padding dropped (all of them are kept when no more than k are real), and
// every selection pass reads them there; otherwise each pass reads them from
// global memory.
// Dynamic smem per warp: 256 words of histogram + kpow2 u64 sort buffer +
// cache_cap u64 cache.
__global__ void merge_topk_kernel(const uint2* __restrict__ cand, uint32_t nq, uint32_t lists,
                                  uint32_t k, uint32_t len, uint64_t stride_q, uint64_t stride_l, uint32_t kpow2,
                                  uint32_t cache_cap, uint32_t sub, uint32_t lists_last, int metric,
                                  float* __restrict__ out_dist, int64_t* __restrict__ out_rows,
                                  uint2* __restrict__ out_cand) {
    extern __shared__ uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t warps = blockDim.x >> 5;
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem) + warp * 256u;
    unsigned long long* buf =
        reinterpret_cast<unsigned long long*>(smem + warps * 1024u) + static_cast<size_t>(warp) * kpow2;
    unsigned long long* cache = reinterpret_cast<unsigned long long*>(smem + warps * 1024u) +
                                static_cast<size_t>(warps) * kpow2 + static_cast<size_t>(warp) * cache_cap;
    const uint32_t q = blockIdx.x * warps + warp;  // output row: query, or (query, group)
    if (q >= nq * sub) return;
    const uint32_t qq = q / sub, grp = q - qq * sub;
    const uint32_t my_lists = grp + 1u == sub ? lists_last : lists;
    const uint2* base = cand + qq * stride_q + static_cast<uint64_t>(grp) * lists * stride_l;
    const uint32_t count = my_lists * len;
    const uint32_t take = min(k, count);
    uint32_t w = 0;
    if (take > 0) {
        if (count <= cache_cap) {
            // Only real candidates enter the cache (padding, row all ones,
            // is dropped here), so the selection passes walk the real ones:
            // lists from shards that own few of a query's probes, or
            // published shorter than their slot, are mostly padding.
            const uint32_t lt = lanemask_lt();
            uint32_t fill = 0;
            auto put = [&](uint2 e) {
                const bool real = e.y != 0xFFFFFFFFu;
                const uint32_t m = __ballot_sync(0xffffffffu, real);
                if (real) cache[fill + __popc(m & lt)] = merge_composite(e);
                fill += __popc(m);
            };
            const uint2 none = make_uint2(0x7f800000u, 0xFFFFFFFFu);
            if (stride_l == len && (reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
                const uint4* src = reinterpret_cast<const uint4*>(base);
                const uint32_t pairs = count / 2u;
                for (uint32_t i0 = 0; i0 < pairs; i0 += 128) {
                    uint4 v[4];
#pragma unroll
                    for (uint32_t u = 0; u < 4; ++u) {
                        const uint32_t i = i0 + u * 32u + lane;
                        v[u] = i < pairs ? src[i] : make_uint4(none.x, none.y, none.x, none.y);
                    }
#pragma unroll
                    for (uint32_t u = 0; u < 4; ++u) {
                        put(make_uint2(v[u].x, v[u].y));
                        put(make_uint2(v[u].z, v[u].w));
                    }
                }
                if (count & 1u) put(lane == 0 ? base[count - 1u] : none);
            } else {
                for (uint32_t j0 = 0; j0 < count; j0 += 128) {
                    uint2 v[4];
#pragma unroll
                    for (uint32_t u = 0; u < 4; ++u) {
                        const uint32_t j = j0 + u * 32u + lane;
                        const uint32_t l = j / len, i = j - l * len;
                        v[u] = j < count ? base[l * stride_l + i] : none;
                    }
#pragma unroll
                    for (uint32_t u = 0; u < 4; ++u) put(v[u]);
                }
            }
            __syncwarp();
            if (fill <= take) {  // every real candidate is kept
                for (uint32_t j = lane; j < fill; j += 32) buf[j] = cache[j];
                w = fill;
            } else {
                w = merge_select([&](uint32_t j) -> unsigned long long { return cache[j]; }, fill, take, hist, buf);
            }
        } else {
            w = merge_select(
                [&](uint32_t idx) -> unsigned long long {
                    const uint32_t l = idx / len, i = idx - l * len;
                    return merge_composite(base[l * stride_l + i]);
                },
                count, take, hist, buf);
        }
    }
    for (uint32_t i = w + lane; i < kpow2; i += 32) buf[i] = ~0ull;
    __syncwarp();
    warp_bitonic_sort(buf, kpow2);
    for (uint32_t i = lane; i < k; i += 32) {
        const unsigned long long c = i < w ? buf[i] : ~0ull;
        const uint32_t row = static_cast<uint32_t>(c & 0xFFFFFFFFull);
        const float key = key_to_float(static_cast<uint32_t>(c >> 32));
        const bool valid = row != 0xFFFFFFFFu;
        if (out_dist != nullptr) {
            float dist = key;
            if (metric == 1) dist = sqrtf(fmaxf(key, 0.0f));
            out_dist[static_cast<size_t>(q) * k + i] = valid ? dist : __int_as_float(0x7f800000);
            out_rows[static_cast<size_t>(q) * k + i] = valid ? static_cast<int64_t>(row) : -1;
        }
        if (out_cand != nullptr) {
            out_cand[static_cast<size_t>(q) * k + i] =
                valid ? make_uint2(__float_as_uint(key), row) : make_uint2(0x7f800000u, 0xFFFFFFFFu);
        }
    }
}

// One warp per row of a distance matrix: the k smallest (value, index) of
// dist[q][0..nb), sorted, padded with {index 0xFFFFFFFF, +inf}. Values of
// +inf and NaN are never taken, as the block top-k's strict "< threshold"
// offer never takes them, so both kernels return the same rows. The row is
// read from global memory (L2) by every selection pass. Dynamic smem per
// warp: 256 words of histogram + kpow2 u64 sort buffer.
__global__ void topk_rows_warp_kernel(const float* __restrict__ dist, uint32_t nq, uint32_t nb, uint32_t k,
                                      uint32_t kpow2, uint32_t* __restrict__ idx_out,
                                      float* __restrict__ val_out) {
    extern __shared__ uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t warps = blockDim.x >> 5;
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem) + warp * 256u;
    unsigned long long* buf =
        reinterpret_cast<unsigned long long*>(smem + warps * 1024u) + static_cast<size_t>(warp) * kpow2;
    const uint32_t q = blockIdx.x * warps + warp;
    if (q >= nq) return;
    const float* row = dist + static_cast<size_t>(q) * nb;
    uint32_t w = 0;
    if (nb > 0) {
        w = merge_select(
            [&](uint32_t j) -> unsigned long long {
                const float v = __ldg(row + j);
                return v < __int_as_float(0x7f800000)
                           ? (static_cast<unsigned long long>(ordered_key(v)) << 32) | j
                           : ~0ull;
            },
            nb, min(k, nb), hist, buf);
    }
    for (uint32_t i = w + lane; i < kpow2; i += 32) buf[i] = ~0ull;
    __syncwarp();
    warp_bitonic_sort(buf, kpow2);
    for (uint32_t i = lane; i < k; i += 32) {
        const unsigned long long c = i < w ? buf[i] : ~0ull;
        const uint32_t r = static_cast<uint32_t>(c & 0xFFFFFFFFull);
        const bool valid = r != 0xFFFFFFFFu;
        idx_out[static_cast<size_t>(q) * k + i] = valid ? r : 0xFFFFFFFFu;
        val_out[static_cast<size_t>(q) * k + i] =
            valid ? key_to_float(static_cast<uint32_t>(c >> 32)) : __int_as_float(0x7f800000);
    }
}

// ------------------------------------------------- filtered-subset gathering
// A row filter selecting a small share of the rows (Vault's equality
// candidates, MetadataIndex::exact_candidates) is searched by gathering the
// selected rows into a contiguous buffer first: the fused kernel then reads
// only those rows instead of streaming the whole base and discarding most
// of it in the epilogue.

// Word w of the selection: filter bits ANDed with the live bits, cut at n.
__device__ __forceinline__ uint32_t selected_word(const uint32_t* __restrict__ mask,
                                                  const uint32_t* __restrict__ live, uint32_t n, uint32_t w) {
    uint32_t m = mask[w];
    if (live != nullptr) m &= live[w];
    const uint32_t left = n - w * 32u;
    if (left < 32u) m &= (1u << left) - 1u;
    return m;
}

// Selected-row listing in two launches over blocks of kSelectThreads words.
constexpr uint32_t kSelectThreads = 256;

// Block-wide exclusive scan of one value per thread (kSelectThreads threads);
// *block_total receives the sum.
__device__ __forceinline__ uint32_t select_block_scan(uint32_t v, uint32_t* warp_sums, uint32_t* block_total) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (uint32_t off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        constexpr uint32_t kWarps = kSelectThreads / 32;
        const uint32_t x = lane < kWarps ? warp_sums[lane] : 0u;
        uint32_t xi = x;
#pragma unroll
        for (uint32_t off = 1; off < 32; off <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, xi, off);
            if (lane >= off) xi += t;
        }
        if (lane < kWarps) warp_sums[lane] = xi - x;
        if (lane == 31) *block_total = xi;
    }
    __syncthreads();
    return warp_sums[warp] + incl - v;
}

// Launch 1: selected rows per block of kSelectThreads words.
__global__ void __launch_bounds__(kSelectThreads) select_count_kernel(const uint32_t* __restrict__ mask,
                                                                      const uint32_t* __restrict__ live, uint32_t n,
                                                                      uint32_t nwords, uint32_t* __restrict__ block_counts) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t total;
    const uint32_t w = blockIdx.x * kSelectThreads + threadIdx.x;
    const uint32_t c = w < nwords ? __popc(selected_word(mask, live, n, w)) : 0u;
    select_block_scan(c, warp_sums, &total);
    if (threadIdx.x == 0) block_counts[blockIdx.x] = total;
}

// Launch 2: each block offsets its rows by the counts of the blocks before
// it, then writes its selected rows in ascending order (at most `cap` rows in
// all); the last block writes the total to *total_out.
__global__ void __launch_bounds__(kSelectThreads) select_rows_kernel(const uint32_t* __restrict__ mask,
                                                                     const uint32_t* __restrict__ live, uint32_t n,
                                                                     uint32_t nwords,
                                                                     const uint32_t* __restrict__ block_counts,
                                                                     uint32_t* __restrict__ rows_out, uint32_t cap,
                                                                     uint32_t* __restrict__ total_out) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t total, before;
    // rows selected by the earlier blocks (a block-wide sum over block_counts)
    uint32_t part = 0;
    for (uint32_t b = threadIdx.x; b < blockIdx.x; b += kSelectThreads) part += block_counts[b];
    select_block_scan(part, warp_sums, &before);
    const uint32_t w = blockIdx.x * kSelectThreads + threadIdx.x;
    uint32_t m = w < nwords ? selected_word(mask, live, n, w) : 0u;
    uint32_t o = before + select_block_scan(__popc(m), warp_sums, &total);
    if (blockIdx.x + 1 == gridDim.x && threadIdx.x == 0) *total_out = before + total;
    while (m != 0u && o < cap) {
        rows_out[o++] = w * 32u + (__ffs(m) - 1u);
        m &= m - 1u;
    }
}

// Selected rows per warp of gather_rows_kernel, and 16-byte loads a lane
// keeps in flight before its stores.
constexpr uint32_t kGatherRowsPerWarp = 4;
constexpr uint32_t kGatherLoadsPerLane = 8;

// One warp per kGatherRowsPerWarp selected rows: copies their operand rows
// (row_bytes, a multiple of 16) and, when norms is given, their squared
// norms. The warp's rows are one flat run of 16-byte chunks; every lane
// issues up to kGatherLoadsPerLane loads before storing them, so a warp has
// whole rows in flight rather than one load per lane.
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                   const uint32_t* __restrict__ rows, uint32_t m, uint32_t row_bytes,
                                   const float* __restrict__ norms, float* __restrict__ norms_out) {
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t r0 = warp * kGatherRowsPerWarp;
    if (r0 >= m) return;
    const uint32_t nr = min(kGatherRowsPerWarp, m - r0);
    const uint32_t my_src = lane < nr ? rows[r0 + lane] : 0u;
    if (norms != nullptr && lane < nr) norms_out[r0 + lane] = norms[my_src];
    const uint32_t chunks = row_bytes / 16u, total = nr * chunks;
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst) + static_cast<size_t>(r0) * chunks;
    for (uint32_t base = 0; base < total; base += 32u * kGatherLoadsPerLane) {
        uint4 v[kGatherLoadsPerLane];
#pragma unroll
        for (uint32_t u = 0; u < kGatherLoadsPerLane; ++u) {
            const uint32_t f = base + u * 32u + lane;
            const uint32_t rr = f / chunks;
            const uint32_t sr = __shfl_sync(0xffffffffu, my_src, rr & 31u);
            if (f < total) v[u] = __ldg(s + static_cast<size_t>(sr) * chunks + (f - rr * chunks));
        }
#pragma unroll
        for (uint32_t u = 0; u < kGatherLoadsPerLane; ++u) {
            const uint32_t f = base + u * 32u + lane;
            if (f < total) d[f] = v[u];
        }
    }
}

// Rows of a search over the gathered subset back to index slots (+ offset):
// out_rows (int64, -1 = none) and/or candidate pairs (row word, all ones = none).
__global__ void remap_rows_kernel(int64_t* __restrict__ out_rows, uint2* __restrict__ out_cand, size_t count,
                                  const uint32_t* __restrict__ rows, uint32_t row_offset) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    if (out_rows != nullptr) {
        const int64_t r = out_rows[i];
        if (r >= 0) out_rows[i] = static_cast<int64_t>(rows[r]) + row_offset;
    }
    if (out_cand != nullptr) {
        const uint32_t r = out_cand[i].y;
        if (r != 0xFFFFFFFFu) out_cand[i].y = rows[r] + row_offset;
    }
}

}  // namespace eb
