// lc_tcgen05.cuh - 5th-generation tensor core (tcgen05) and tensor memory
// (TMEM) helpers for sm_100a: allocation, shared-memory matrix descriptors,
// the bf16 MMA with fp32 accumulation in TMEM, commits to mbarriers, and
// TMEM <-> register moves. Used by the causal prefill kernel.
#pragma once

#include "lc_common.cuh"

namespace lc {

// ------------------------------------------------------------------ TMEM ----
// Allocates `ncols` TMEM columns (power of two >= 32) for this CTA; one whole
// warp executes it; the TMEM address is written to *smem_dst.
__device__ inline void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ inline void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Orders tcgen05 operations around thread synchronisation (mbarrier waits,
// barriers): "before" ahead of the arrive, "after" behind the wait.
__device__ inline void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ inline void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor-core operand reads, TMA).
__device__ inline void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------- descriptors --
// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile (the
// layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B; tiles 1024-byte aligned).
//   K-major (rows of 64 bf16 = 128 B, 8-row groups 1024 B apart):
//       lbo = 16, sbo = 1024
//   MN-major (64 contiguous elements = 128 B per K row; 8 K rows per 1024 B
//   group; the next 64-element MN block `lbo` bytes further):
//       lbo = distance between MN blocks, sbo = 1024
// Fields: start address >> 4 (bits 0-13), leading byte offset >> 4 (16-29),
// stride byte offset >> 4 (32-45), version 1 (46-47), base offset 0,
// layout type 2 = 128-byte swizzle (61-63).
__device__ inline uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B, fp32 D,
// M x N, A K-major, B K-major (b_mn_major = 0) or MN-major (1).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int b_mn_major) {
    return (1u << 4)                            // D format: f32
           | (1u << 7)                          // A format: bf16
           | (1u << 10)                         // B format: bf16
           | ((uint32_t)b_mn_major << 16)       // B major
           | ((uint32_t)(N >> 3) << 17)         // N / 8
           | ((uint32_t)(M >> 4) << 24);        // M / 16
}

// ------------------------------------------------------------------- MMA ----
// D[tmem] (+)= A[smem] * B[smem]^T, one elected thread issues it.
__device__ inline void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A (M rows = TMEM lanes, K-major, two bf16
// per 32-bit column) read from tensor memory.
__device__ inline void umma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives (once) on `bar` when every tcgen05 operation this thread issued so
// far has completed.
__device__ inline void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// ------------------------------------------------------ TMEM <-> registers --
// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (quadrant base + i), columns [col, col + 32).
__device__ inline void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
        "%30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ inline void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from registers.
__device__ inline void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

__device__ inline void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// tcgen05.wait::ld that also ties the 32 destination registers of an earlier
// tmem_ld32, so that the compiler cannot move their uses above the wait.
__device__ inline void tmem_wait_ld_regs(uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
          "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
          "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
          "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
          "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
        :
        : "memory");
}
__device__ inline void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }


// ------------------------------------------------------- CTA pairs (2-SM) --
// A cluster of two CTAs on neighbouring SMs sharing one tcgen05.mma: each CTA
// holds half of A (M/2 rows) and half of B (N/2 rows) in its shared memory and
// receives its M/2 rows of D in its own TMEM. Rank 0 issues the MMAs.

__device__ inline uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of `local` (a shared::cta address) in CTA `rank`.
__device__ inline uint32_t mapa_shared(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

// Every thread of both CTAs: release its prior accesses, wait for the other CTA.
__device__ inline void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
// The two halves of cluster_sync, for work in between: every thread of the
// cluster arrives once, then waits once.
__device__ inline void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ inline void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ inline void tmem_alloc_2sm(uint32_t *smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ inline void tmem_relinquish_2sm() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ inline void tmem_dealloc_2sm(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// D[tmem of both CTAs] (+)= A . B^T over the pair (M = 256 in the descriptor).
__device__ inline void umma_bf16_2sm(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                     uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` (same shared-memory offset) in each CTA of `cta_mask`
// when the pair's MMAs issued so far have completed.
__device__ inline void umma_commit_2sm(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
        "[%0], %1;" ::"r"(smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

// Tiled load into this CTA's shared memory whose byte count completes on an
// mbarrier of either CTA of the pair (`bar_cluster`: shared::cluster address).
// No multicast: each CTA fetches only its own half of each operand.
__device__ inline void tma_load_2d_2sm(void *smem_dst, const CUtensorMap *map, int x, int y,
                                       uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}

// Arrive on an mbarrier of either CTA of the cluster (release at cluster scope).
__device__ inline void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
                 : "memory");
}

// try_wait with acquire at cluster scope (arrivals from the other CTA).
__device__ inline bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ inline bool mbar_wait_bounded_cluster(uint64_t *bar, uint32_t parity,
                                                 volatile int *abort_flag, int *status) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                *abort_flag = 1;
                set_status(status, LC_DEV_TIMEOUT);
                return false;
            }
        }
    }
}

}  // namespace lc
