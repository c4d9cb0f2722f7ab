// Warp-cooperative k-selection over candidate lists held in global memory.
//
// A candidate is a uint2 {float key bits, row}. Lists are kept in ascending
// row order (candidates are appended in scan order and every compaction below
// is stable), so "ascending (key, row)" order equals "ascending key, earlier
// position first" and a 32-bit radix select on the key plus a stable
// tie-break by position reproduces the (key, row) order exactly.
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace eb {

// Finds the k-th smallest ordered key (1-based rank k) among list[0, count)
// with a 4-pass, 8-bit radix select. hist is a 256-word shared-memory scratch
// owned by this warp. On return *kth_key is the ordered key of rank k and
// *need_eq is how many entries equal to it belong to the k smallest.
// Requires 1 <= k <= count. Must be called by the whole warp.
__device__ __forceinline__ void warp_radix_select(const uint2* list, uint32_t count, uint32_t k,
                                                  uint32_t* hist, uint32_t* kth_key,
                                                  uint32_t* need_eq) {
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t prefix = 0, prefix_mask = 0, rank = k;
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
        const uint32_t shift = 24u - 8u * static_cast<uint32_t>(pass);
        for (uint32_t b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
        for (uint32_t j = lane; j < count; j += 32) {
            const uint32_t u = ordered_key(__uint_as_float(list[j].x));
            if ((u & prefix_mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
        }
        __syncwarp();
        // lane owns bins [8*lane, 8*lane + 8)
        uint32_t bins[8];
        uint32_t local = 0;
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
        uint32_t digit = 0, before = excl;
        if (mine) {
            uint32_t acc = excl;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (acc + bins[i] >= rank) {
                    digit = lane * 8 + i;
                    before = acc;
                    break;
                }
                acc += bins[i];
            }
        }
        const uint32_t owner = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
        digit = __shfl_sync(0xffffffffu, digit, owner);
        before = __shfl_sync(0xffffffffu, before, owner);
        rank -= before;
        prefix |= digit << shift;
        prefix_mask |= 255u << shift;
        __syncwarp();
    }
    *kth_key = prefix;
    *need_eq = rank;
}

// Stable in-place compaction of list[0, count) down to its k smallest
// (key, position) entries. Returns the float key of rank k (the new admission
// threshold: later candidates need key < threshold). Whole warp.
__device__ __forceinline__ float warp_compact_list(uint2* list, uint32_t count, uint32_t k,
                                                   uint32_t* hist) {
    uint32_t kth, need_eq;
    warp_radix_select(list, count, k, hist, &kth, &need_eq);
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t lt_mask = lanemask_lt();
    uint32_t w = 0, eq_taken = 0;
    for (uint32_t j0 = 0; j0 < count; j0 += 32) {
        const uint32_t j = j0 + lane;
        uint2 e = make_uint2(0u, 0u);
        if (j < count) e = list[j];
        const uint32_t u = ordered_key(__uint_as_float(e.x));
        const bool lt = j < count && u < kth;
        const bool eq = j < count && u == kth;
        const uint32_t eq_mask = __ballot_sync(0xffffffffu, eq);
        const uint32_t eq_rank = eq_taken + __popc(eq_mask & lt_mask);
        const bool keep = lt || (eq && eq_rank < need_eq);
        const uint32_t keep_mask = __ballot_sync(0xffffffffu, keep);
        if (keep) list[w + __popc(keep_mask & lt_mask)] = e;
        w += __popc(keep_mask);
        eq_taken += __popc(eq_mask);
    }
    __syncwarp();
    return key_to_float(kth);
}

// Same contract as warp_compact_list for count <= 32*E, with the list held in
// registers for the whole selection: one batch of independent loads, radix
// passes over registers, one stable write-back. Entry j of the list lives in
// slot j/32 of lane j%32, so the write-back walks positions in order.
// The passes start at the first byte in which the keys differ (a list's keys
// share their high bytes, and a pass over a shared byte only piles every
// entry onto one histogram bin), and stop early once the bin holding rank k
// is taken whole; the threshold is then that bin's largest key.
template <int E>
__device__ __forceinline__ float warp_compact_regs(uint2* list, uint32_t count, uint32_t k,
                                                   uint32_t* hist) {
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t key[E], row[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const uint32_t j = static_cast<uint32_t>(i) * 32u + lane;
        uint2 e = make_uint2(0u, 0u);
        if (j < count) e = list[j];
        key[i] = ordered_key(__uint_as_float(e.x));
        row[i] = e.y;
    }
    // Bytes shared by every entry (entry 0 exists: count >= k >= 1).
    const uint32_t key0 = __shfl_sync(0xffffffffu, key[0], 0);
    uint32_t diff = 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const uint32_t j = static_cast<uint32_t>(i) * 32u + lane;
        if (j < count) diff |= key[i] ^ key0;
    }
    diff = __reduce_or_sync(0xffffffffu, diff);
    const int first = diff == 0u ? 4 : static_cast<int>(__clz(diff) >> 3);
    uint32_t pmask = first == 0 ? 0u : (first >= 4 ? 0xFFFFFFFFu : (0xFFFFFFFFu << (32 - 8 * first)));
    uint32_t prefix = key0 & pmask, rank = k;
#pragma unroll 1
    for (int pass = first; pass < 4; ++pass) {
        const uint32_t shift = 24u - 8u * static_cast<uint32_t>(pass);
        for (uint32_t b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < E; ++i) {
            const uint32_t j = static_cast<uint32_t>(i) * 32u + lane;
            if (j < count && (key[i] & pmask) == prefix) atomicAdd(&hist[(key[i] >> shift) & 255u], 1u);
        }
        __syncwarp();
        uint32_t bins[8];
        uint32_t local = 0;
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
        prefix |= digit << shift;
        pmask |= 255u << shift;
        __syncwarp();
        if (inbin == rank) break;  // the whole bin is selected
    }
    // Keep every entry below the selected group and the first `rank` entries
    // of the group (all of it after an early stop).
    uint32_t kth = prefix;
    if (pmask != 0xFFFFFFFFu) {
        uint32_t mx = 0;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            const uint32_t j = static_cast<uint32_t>(i) * 32u + lane;
            if (j < count && (key[i] & pmask) == prefix) mx = max(mx, key[i]);
        }
        kth = __reduce_max_sync(0xffffffffu, mx);
    }
    const uint32_t need_eq = rank;
    const uint32_t lt_mask = lanemask_lt();
    uint32_t w = 0, eq_taken = 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const uint32_t j = static_cast<uint32_t>(i) * 32u + lane;
        const bool valid = j < count;
        const uint32_t km = key[i] & pmask;
        const bool lt = valid && km < prefix;
        const bool eq = valid && km == prefix;
        const uint32_t eq_mask = __ballot_sync(0xffffffffu, eq);
        const uint32_t eq_rank = eq_taken + __popc(eq_mask & lt_mask);
        const bool keep = lt || (eq && eq_rank < need_eq);
        const uint32_t keep_mask = __ballot_sync(0xffffffffu, keep);
        if (keep) list[w + __popc(keep_mask & lt_mask)] = make_uint2(__float_as_uint(key_to_float(key[i])), row[i]);
        w += __popc(keep_mask);
        eq_taken += __popc(eq_mask);
    }
    __syncwarp();
    return key_to_float(kth);
}

}  // namespace eb
