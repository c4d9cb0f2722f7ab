// Inline-PTX wrappers for the sm_100a features the search kernels use:
// mbarriers, TMA tiled loads, tcgen05 (TMEM alloc, MMA, commit, TMEM loads),
// and the bounded waits every spin in this library goes through.
//
// Every wait is bounded: after kWaitTimeoutCycles the waiting thread records
// an error code in the device-global error word and raises the CTA's abort
// flag, so a pipeline that loses a producer or consumer returns with an error
// status instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace eb {

// Device-global error word (0 = ok). Written with atomicCAS so the first error
// wins; read and cleared by the host through read_and_clear_device_error().
// All device code of the library is compiled in one translation unit
// (engine.cu), so this internal-linkage definition is the only instance.
static __device__ int g_device_error = 0;

enum DeviceError : int {
    kDevErrNone = 0,
    kDevErrWaitTimeout = 1,      // a bounded mbarrier wait expired
    kDevErrBadConfig = 2,        // a launch was given a shape it cannot handle
};

// ~1.1 s at 1.9 GHz. Healthy waits in these kernels last microseconds.
constexpr long long kWaitTimeoutCycles = 1LL << 31;

__device__ __forceinline__ void record_device_error(int code) {
    atomicCAS(&g_device_error, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete, for at most `budget`
// cycles. Returns false (and raises *abort) if the wait expired or another
// role already aborted.
__device__ __forceinline__ bool mbar_wait_for(uint32_t bar, uint32_t parity, volatile int* abort,
                                              long long budget) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (clock64() - start > budget) {
            record_device_error(kDevErrWaitTimeout);
            *abort = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    return mbar_wait_for(bar, parity, abort, kWaitTimeoutCycles);
}

// ---------------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load into this CTA's shared memory; completion is signalled on
// `bar` as transaction bytes. x is the innermost (contiguous) coordinate in
// elements and is always a multiple of 128 bytes here.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// ------------------------------------------------------------ CTA pairs
// A CTA pair is a cluster of two CTAs whose MMAs run as one (cta_group::2):
// rank 0 issues them over both CTAs' shared memory and both CTAs' TMEM.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_count_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// Address of the same shared-memory object in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// Every thread of both CTAs: arrive (release) and wait (acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier that may live in another CTA of the cluster. The
// release is CTA-scoped: the arrival hands over a TMEM accumulator (ordered
// by tcgen05.fence::before_thread_sync), not memory written for the peer, so
// it need not wait for this thread's outstanding global stores to reach L2.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait for a barrier that also receives arrivals from the peer CTA.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (*abort) return false;
        if (clock64() - start > kWaitTimeoutCycles) {
            record_device_error(kDevErrWaitTimeout);
            *abort = 1;
            return false;
        }
    }
    return true;
}

// 2-D tiled load of one CTA's half of a pair operand into its own shared
// memory, completion signalled on rank 0's barrier (`bar_cluster`, a
// shared::cluster address). No multicast: each CTA fetches its own half.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}

// ------------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Makes `bar` track completion of every tcgen05.mma this thread issued before.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// Pair (cta_group::2) forms: both CTAs' warp 1 allocate / free together
// (same columns in both TMEMs); rank 0 issues the MMAs and commits.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Completion of this thread's pair MMAs arrives once on the barrier at the
// same offset in every CTA of `cta_mask` (this is an mbarrier signal from the
// tensor core, not a memory load).
__device__ __forceinline__ void tc_commit_pair_both(uint32_t bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"(cta_mask)
        : "memory");
}

__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

enum class MmaKind { F16, TF32, I8 };

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, one instruction, issued by one
// thread. `accumulate` = 0 overwrites D. CG = 2: the pair form, M = 256 over
// both CTAs' A halves and N over both CTAs' B halves.
template <MmaKind K, int CG = 1>
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
#define EB_TC_MMA(GROUP, KINDSTR)                                                              \
    asm volatile(                                                                             \
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"                                   \
        "tcgen05.mma.cta_group::" GROUP ".kind::" KINDSTR " [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d), \
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)                                    \
        : "memory")
    if constexpr (CG == 1) {
        if constexpr (K == MmaKind::F16) EB_TC_MMA("1", "f16");
        else if constexpr (K == MmaKind::TF32) EB_TC_MMA("1", "tf32");
        else EB_TC_MMA("1", "i8");
    } else {
        if constexpr (K == MmaKind::F16) EB_TC_MMA("2", "f16");
        else if constexpr (K == MmaKind::TF32) EB_TC_MMA("2", "tf32");
        else EB_TC_MMA("2", "i8");
    }
#undef EB_TC_MMA
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle that TMA's CU_TENSOR_MAP_SWIZZLE_128B writes: rows of 128
// bytes, 8-row atoms of 1024 bytes stacked along M/N. Fields: start address
// >> 4 (bits 0-13), leading byte offset >> 4 (16-29; unused for swizzled
// K-major, 1 by convention), stride byte offset >> 4 (32-45; 1024 bytes
// between 8-row atoms), descriptor version 1 (bit 46), swizzle mode 2 =
// 128-byte (bits 61-63). The tile base must be 1024-byte aligned; stepping K
// inside the atom is a plain +32-byte start-address offset.
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor (32-bit) for a dense, K-major x K-major MMA.
//   c_fmt: 0 f16, 1 f32, 2 s32 (bits 4-5)
//   ab_fmt: kind::f16 -> 0 f16, 1 bf16; kind::tf32 -> 2; kind::i8 -> 1 signed
//   (bits 7-9 for A, 10-12 for B); N >> 3 at bits 17-22; M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t ab_fmt, uint32_t m,
                                                  uint32_t n) {
    return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// 32 lanes x 32 columns of 32-bit TMEM words into 32 registers per thread.
// Thread t of the warp reads lane (lane base of taddr) + t. The instruction is
// .sync.aligned: every lane of the warp must execute it together, so callers
// place a __syncwarp() directly before it after any lane-dependent branch.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
        " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
        " [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


// ------------------------------------------------------------ misc helpers

// Global 8-byte store executed only where `pred` holds, as a predicated
// instruction: a per-lane condition never becomes a divergent branch.
__device__ __forceinline__ void st_global_pred(uint2* addr, uint32_t x, uint32_t y, bool pred) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %3, 0;\n\t"
        "@p st.global.v2.u32 [%0], {%1, %2};\n\t}"
        :
        : "l"(addr), "r"(x), "r"(y), "r"(pred ? 1u : 0u)
        : "memory");
}

__device__ __forceinline__ bool elect_one_sync() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
        "elect.sync r|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// Order-preserving map float -> uint32 (ascending floats -> ascending uints).
__device__ __forceinline__ uint32_t ordered_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return b ^ ((b & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t u) {
    const uint32_t b = u ^ ((u & 0x80000000u) ? 0x80000000u : 0xFFFFFFFFu);
    return __uint_as_float(b);
}

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

}  // namespace eb
