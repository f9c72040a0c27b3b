// lc_common.cuh - device helpers shared by the sm_100a kernels of the paged
// attention path: bf16 packing, the paged-pool address rule, mbarrier waits
// with a time bound, TMA tile loads, ldmatrix / mma.sync / movmatrix wrappers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lucciola_attn.h"

namespace lc {

typedef __nv_bfloat16 bf16;

constexpr int kBlockSize = 16;  // tokens per page (src/layers/kv_cache.rs:35)

// Row index of (physical block, layer, kv head) in a pool viewed as a 2-D
// [num_blocks*num_layers*num_kv_heads*16][head_dim] matrix; token t of the page
// is row + t. Same strides as src/kernels/kv_cache.cu:39-48.
__host__ __device__ inline int64_t page_row(int64_t phys, int layer, int kv_head,
                                            int num_layers, int num_kv_heads) {
    return ((phys * num_layers + layer) * num_kv_heads + kv_head) * kBlockSize;
}

__device__ inline void set_status(int *status, int bits) {
    if (status) atomicOr(status, bits);
}

// Atomic add with acquire-release semantics at GPU scope; returns the old value.
__device__ inline int atom_add_acq_rel_gpu(int *addr, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
    return old;
}

__device__ inline uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ inline uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch (sm_90+): both are no-ops for a grid that was
// not launched with programmatic stream serialization.
__device__ inline void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ inline void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier --
__device__ inline void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ inline void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ inline void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ inline void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ inline bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar` to complete, for at most kWaitLimitNs.
// `abort_flag` (shared) lets one timed-out thread release every other waiter of
// the CTA. Returns false on timeout (after setting the flag and the status bit).
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ inline bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                         volatile int *abort_flag, int *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
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

// After a wait gave up: waits (bounded again) for a phase whose copies may
// still be in flight, so that the CTA does not exit under them.
__device__ inline void mbar_wait_drain(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - t0 > kWaitLimitNs) return;
}

// ------------------------------------------------------------------- TMA ----
// 2-D tiled bulk tensor load into this CTA's shared memory, completion counted
// on `bar` in bytes. x (innermost) must keep x*2 bytes 16-byte aligned: every
// call site passes x = 0 or 64.
__device__ inline void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                   uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ inline void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------ warp MMA -----
__device__ inline void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ inline void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ inline void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                      uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transposes an 8x8 matrix of 16-bit values held one row-pair per lane.
__device__ inline uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ inline uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ inline void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace lc
