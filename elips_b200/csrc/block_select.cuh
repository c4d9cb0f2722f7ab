// Block-level running top-k for the SIMT scan kernels (quantized scans, the
// GpuPort primitives, IVF-PQ). A CTA streams candidates (key, row) in
// ascending row order; candidates below the admission threshold are appended
// to a shared-memory buffer, which is compacted to the k smallest
// (key, row) pairs whenever another round could overflow it. The k-th key
// then becomes the threshold (strict: a later candidate with an equal key has
// a larger row and ranks after the kept one).
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace eb {

// Shared-memory state of one running top-k. `cap` >= k + threads.
struct BlockTopK {
    uint2* buf;      // [cap] {key bits, row}
    uint2* tmp;      // [cap] compaction target
    uint32_t* hist;  // [256]
    uint32_t* cnt;   // [1]
    float* thr;      // [1]
    uint32_t* sel;   // [4] scratch: digit, before, kept
    uint32_t cap;
};

__device__ __forceinline__ unsigned long long composite_of(uint2 e) {
    return (static_cast<unsigned long long>(ordered_key(__uint_as_float(e.x))) << 32) | e.y;
}

__device__ __forceinline__ void btk_init(const BlockTopK& s) {
    if (threadIdx.x == 0) {
        *s.cnt = 0;
        *s.thr = __int_as_float(0x7f800000);
    }
    __syncthreads();
}

// Every thread of the block calls this once per round (has = false for no
// candidate). Ends with a barrier.
__device__ __forceinline__ void btk_offer(const BlockTopK& s, bool has, float key, uint32_t row) {
    if (has && key < *s.thr) {
        const uint32_t pos = atomicAdd(s.cnt, 1u);
        s.buf[pos] = make_uint2(__float_as_uint(key), row);
    }
    __syncthreads();
}

// Reduces the buffer to its k smallest composites (unique: rows are unique).
// Whole block; ends with a barrier.
__device__ __forceinline__ void btk_compact(const BlockTopK& s, uint32_t k) {
    const uint32_t count = *s.cnt;
    if (count <= k) return;
    unsigned long long prefix = 0, pmask = 0;
    uint32_t rank = k;
    for (int pass = 0; pass < 8; ++pass) {
        const uint32_t shift = 56u - 8u * static_cast<uint32_t>(pass);
        for (uint32_t b = threadIdx.x; b < 256; b += blockDim.x) s.hist[b] = 0;
        __syncthreads();
        for (uint32_t j = threadIdx.x; j < count; j += blockDim.x) {
            const unsigned long long c = composite_of(s.buf[j]);
            if ((c & pmask) == prefix) atomicAdd(&s.hist[(c >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            const uint32_t lane = threadIdx.x;
            uint32_t bins[8], local = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                bins[i] = s.hist[lane * 8 + i];
                local += bins[i];
            }
            uint32_t incl = local;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= static_cast<uint32_t>(off)) incl += t;
            }
            const uint32_t excl = incl - local;
            if (excl < rank && rank <= incl) {
                uint32_t acc = excl;
                for (int i = 0; i < 8; ++i) {
                    if (acc + bins[i] >= rank) {
                        s.sel[0] = lane * 8 + i;
                        s.sel[1] = acc;
                        break;
                    }
                    acc += bins[i];
                }
            }
        }
        __syncthreads();
        rank -= s.sel[1];
        prefix |= static_cast<unsigned long long>(s.sel[0]) << shift;
        pmask |= 255ull << shift;
        __syncthreads();
    }
    // prefix is the k-th smallest composite: keep everything <= it.
    if (threadIdx.x == 0) s.sel[2] = 0;
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < count; j += blockDim.x) {
        const uint2 e = s.buf[j];
        if (composite_of(e) <= prefix) s.tmp[atomicAdd(&s.sel[2], 1u)] = e;
    }
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < k; j += blockDim.x) s.buf[j] = s.tmp[j];
    if (threadIdx.x == 0) {
        *s.cnt = k;
        *s.thr = key_to_float(static_cast<uint32_t>(prefix >> 32));
    }
    __syncthreads();
}

// Called by the whole block between rounds of `threads` offers.
__device__ __forceinline__ void btk_maybe_compact(const BlockTopK& s, uint32_t k) {
    if (*s.cnt + blockDim.x > s.cap) btk_compact(s, k);
}

// Final: compact to k and write k entries (unsorted, padded) to out.
__device__ __forceinline__ void btk_finish(const BlockTopK& s, uint32_t k, uint2* out) {
    btk_compact(s, k);
    const uint32_t c = *s.cnt;
    for (uint32_t j = threadIdx.x; j < k; j += blockDim.x)
        out[j] = j < c ? s.buf[j] : make_uint2(0x7f800000u, 0xFFFFFFFFu);
    __syncthreads();
}

}  // namespace eb
