// proj_gemm.cu - the projections on either side of attention, on the 5th-gen
// tensor cores: out[M][N] = x[M][K] . w[N][K]^T with fp32 accumulation in
// tensor memory and a bf16 result, as Qwen2Model::matmul_bf16 computes it
// (src/models.rs:252-292: cublasGemmEx, CUBLAS_COMPUTE_32F, bf16 C). Three
// epilogues:
//   plain     out = bf16(acc)                                  (qkv_proj, beta 0)
//   residual  out = bf16(acc + residual)                       (o_proj, beta 1,
//             src/models.rs:553-566; residual may be out itself)
//   qkv rope  the QKV projection followed, in the same kernel, by what
//             lc_rope_append does to its rows (src/models.rs:500-534): q and
//             k rounded to bf16, bias added, rotated and stored back; k
//             rotated and v + bias appended to the paged pools. The result is
//             bit-identical to lc_proj_gemm then lc_rope_append.
//
// Design (M > 128 token rows, a prompt): a persistent grid of CTA pairs walks
// 256 x 256 output tiles (the 256 columns of a tile hold whole heads:
// head_dim 64 or 128); see the CTA-pair section below. A decode step's
// M <= 128 rows go to the weight-streaming kernel of proj_decode.cu. In the
// pair kernel warp 0 issues TMA loads of 64-wide K blocks (128-byte swizzle)
// into the stage ring; warp 1 issues tcgen05.mma (bf16 in, fp32 accumulate)
// into one of two 256-column TMEM accumulators; warps 2-9 (one output row per
// thread of a TMEM lane quadrant) drain the other accumulator through the
// epilogue while the next tile accumulates (two warps per quadrant, each
// taking every other 32-column chunk or head, so that one warp's loads
// overlap the other's arithmetic). Every wait is bounded; a timeout sets
// LC_DEV_TIMEOUT.
#include <climits>

#include "lc_common.cuh"
#include "lc_host.h"
#include "lc_tcgen05.cuh"
#include "rope_math.cuh"

namespace lc {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kEpiWarps = 8;    // two per TMEM lane quadrant
constexpr int kThreadsG = 64 + 32 * kEpiWarps;  // TMA warp, MMA warp, epilogue warps
constexpr uint32_t kTmemColsG = 2 * kBN;         // two accumulators

enum Epilogue { kPlain = 0, kResidual = 1, kQkvRope = 2 };

struct GemmParams {
    int M, N, K;
    int m_tiles, n_tiles;
    bf16 *out;
    int64_t out_stride;
    const bf16 *residual;
    int64_t res_stride;
    // qkv rope: rows are tokens (row / tokens_per_seq = sequence), columns
    // [q heads | k heads | v heads] of head_dim each.
    int tokens_per_seq;
    const int *positions;
    const bf16 *q_bias, *k_bias, *v_bias;
    const float *cos_t, *sin_t;
    int rope_rows;
    bf16 *k_pool, *v_pool;
    int64_t num_blocks;
    int num_layers, layer, num_q_heads, num_kv_heads, head_dim;
    const int *tables;
    int table_stride;
    int *status;
};

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// bf16(acc) back as a float: the value the reference's qkv buffer holds.
__device__ __forceinline__ float round_bf16(float x) {
    return __bfloat162float(__float2bfloat16(x));
}

// 32 consecutive bf16 from 32 floats (RNE), four 16-byte stores.
__device__ __forceinline__ void store32(bf16 *dst, const float (&f)[32]) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        uint4 o;
        o.x = pack_bf16(f[8 * v + 0], f[8 * v + 1]);
        o.y = pack_bf16(f[8 * v + 2], f[8 * v + 3]);
        o.z = pack_bf16(f[8 * v + 4], f[8 * v + 5]);
        o.w = pack_bf16(f[8 * v + 6], f[8 * v + 7]);
        reinterpret_cast<uint4 *>(dst)[v] = o;
    }
}

// 32 consecutive bf16 as floats.
__device__ __forceinline__ void load32(const bf16 *src, float (&f)[32]) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const uint4 u = reinterpret_cast<const uint4 *>(src)[v];
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[8 * v + 2 * i] = __low2float(h[i]);
            f[8 * v + 2 * i + 1] = __high2float(h[i]);
        }
    }
}

// Pool offset of (position, kv head 0) for token row `row`, or -1 when the
// row must not be appended (status bits set), as rope_append.cu does.
__device__ __forceinline__ int64_t pool_base(const GemmParams &p, int row, int pos) {
    const int b = row / p.tokens_per_seq;
    const int logical = pos / kBlockSize;
    if (logical >= p.table_stride) {
        set_status(p.status, LC_DEV_BAD_POS);
        return -1;
    }
    const int phys = p.tables[(int64_t)b * p.table_stride + logical];
    if (phys < 0 || phys >= p.num_blocks) {
        set_status(p.status, LC_DEV_BAD_BLOCK);
        return -1;
    }
    return page_row(phys, p.layer, 0, p.num_layers, p.num_kv_heads) * p.head_dim +
           (int64_t)(pos % kBlockSize) * p.head_dim;
}

// Output of the epilogue warps: the warp's 32 rows x 32 columns go to shared memory (64-byte rows, 64-byte swizzle as the output
// tensor map has it) and lane 0 writes them with one TMA store per box; two
// buffers of two boxes per warp, so a step's stores overlap the next step.
struct OutStaged {
    uint8_t *base;  // this warp's 8 KiB, 2 KiB aligned
    const CUtensorMap *map;
    int step, lane;
    __device__ __forceinline__ uint8_t *buf(int box) const {
        return base + (step & 1) * 4096 + box * 2048;
    }
    // The buffer about to be written was last stored two steps ago.
    __device__ __forceinline__ void begin() {
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncwarp();
    }
    __device__ __forceinline__ void put(int, bool, int, int box, const float (&f)[32]) {
        uint8_t *b = buf(box) + lane * 64;
        const int sw = (lane >> 1) & 3;  // 64-byte swizzle: 16-byte chunk ^ address bits 7-8
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            uint4 o;
            o.x = pack_bf16(f[8 * v + 0], f[8 * v + 1]);
            o.y = pack_bf16(f[8 * v + 2], f[8 * v + 3]);
            o.z = pack_bf16(f[8 * v + 4], f[8 * v + 5]);
            o.w = pack_bf16(f[8 * v + 6], f[8 * v + 7]);
            *reinterpret_cast<uint4 *>(b + ((v ^ sw) << 4)) = o;
        }
    }
    // Boxes 0 .. nbox-1 of this step go to columns x0 / x1 of rows y .. y + 31.
    __device__ __forceinline__ void issue(int nbox, int x0, int x1, int y, bool any_row) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0 && any_row) {
            for (int b = 0; b < nbox; ++b)
                asm volatile(
                    "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                        reinterpret_cast<uint64_t>(map)),
                    "r"(b ? x1 : x0), "r"(y), "r"(smem_u32(buf(b)))
                    : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        ++step;
    }
    // Before the CTA exits: every store has been written out.
    __device__ __forceinline__ void drain() {
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
};

// Epilogue of one 256-column tile for the thread owning output row `row`
// (TMEM lane quadrant base `tacc`; the warp's rows start at `y`): plain /
// residual; chunks half, half + 2, ...
template <int EPI, class Out>
__device__ __forceinline__ void epilogue_rows(const GemmParams &p, uint32_t tacc, int row, int y,
                                              int col0, int half, Out &o) {
    const bool live = row < p.M;
#pragma unroll 1
    for (int c = half; c < kBN / 32; c += 2) {
        const int col = col0 + 32 * c;
        if (col >= p.N) break;
        uint32_t r[32];
        tmem_ld32(tacc + 32 * c, r);
        tmem_wait_ld_regs(r);
        float f[32];
        if constexpr (EPI == kResidual) {
            float res[32];
            if (live) {
                load32(p.residual + (int64_t)row * p.res_stride + col, res);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) res[i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] = __fadd_rn(u2f(r[i]), res[i]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] = u2f(r[i]);
        }
        o.begin();
        o.put(row, live, col, 0, f);
        o.issue(1, col, 0, y, y < p.M);
    }
}

// What the QKV epilogue needs of a row besides the accumulator, read while
// the tile still accumulates: the position, the 32 cos/sin of the row's RoPE
// chunk (a thread works on one fixed 32-dim chunk of every half head of the
// tile) and the pool offset when the tile holds k or v heads.
template <int HD>
struct QkvRow {
    int pos;
    bool live, rope_ok;
    int64_t base;  // pool offset of (pos, kv head 0), or -1
    float cs[32], sn[32];

    __device__ __forceinline__ void load(const GemmParams &p, int row, int col0, int half) {
        constexpr int kHalf = HD / 2;
        constexpr int kChunks = kHalf / 32;
        live = row < p.M;
        pos = live ? p.positions[row] : 0;
        if (live && pos < 0) set_status(p.status, LC_DEV_BAD_POS);
        rope_ok = live && pos >= 0 && pos < p.rope_rows;
        if (live && pos >= p.rope_rows) set_status(p.status, LC_DEV_BAD_POS);
        base = -1;
        if (live && pos >= 0 && col0 + kBN > p.num_q_heads * HD) base = pool_base(p, row, pos);
        const int d0 = 32 * (kChunks == 1 ? 0 : half);
        const float *ct = p.cos_t + (int64_t)(rope_ok ? pos : 0) * kHalf + d0;
        const float *st = p.sin_t + (int64_t)(rope_ok ? pos : 0) * kHalf + d0;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const float4 c = reinterpret_cast<const float4 *>(ct)[v];
            const float4 n = reinterpret_cast<const float4 *>(st)[v];
            cs[4 * v] = c.x, cs[4 * v + 1] = c.y, cs[4 * v + 2] = c.z, cs[4 * v + 3] = c.w;
            sn[4 * v] = n.x, sn[4 * v + 1] = n.y, sn[4 * v + 2] = n.z, sn[4 * v + 3] = n.w;
        }
    }
};

// QKV epilogue: head by head over the tile's columns (a warp pair splits them:
// 32-dim chunks half, half + 2, ... of the tile's half-heads). Per element the
// arithmetic is that of rope_append_vec_kernel on the bf16-rounded GEMM result;
// the row keeps the projection where rope_append leaves it (v, a negative
// position, a position past the RoPE table).
template <int HD, class Out>
__device__ __forceinline__ void epilogue_qkv(const GemmParams &p, uint32_t tacc, int row, int y,
                                             int col0, int half, const QkvRow<HD> &w, Out &o) {
    constexpr int kHalf = HD / 2;
    const int hq = p.num_q_heads, hkv = p.num_kv_heads;
    const bool live = w.live;
    const int64_t base = w.base;
    const int64_t stride_blk = (int64_t)kBlockSize * HD;
    constexpr int kChunks = kHalf / 32;  // 32-dim chunks per half head
#pragma unroll 1
    for (int hcx = half; hcx < (kBN / HD) * kChunks; hcx += 2) {
        const int h = hcx / kChunks, c = hcx - h * kChunks;
        const int hc = col0 + h * HD;  // first column of this head
        if (hc >= p.N) break;
        const int g = hc / HD;  // head index over [q | k | v]
        const int kind = g < hq ? 0 : (g < hq + hkv ? 1 : 2);
        const int d0 = 32 * c;  // dims [d0, d0 + 32) of the first half, their partners
        uint32_t r1[32], r2[32];
        tmem_ld32(tacc + h * HD + d0, r1);
        tmem_ld32(tacc + h * HD + kHalf + d0, r2);
        tmem_wait_ld_regs(r1);
        tmem_wait_ld_regs(r2);
        float x1[32], x2[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            x1[i] = round_bf16(u2f(r1[i]));
            x2[i] = round_bf16(u2f(r2[i]));
        }
        const bool appendable = live && w.pos >= 0 && base >= 0;
        if (live && w.pos >= 0 && kind != 2 && w.rope_ok) {
            const int hh = kind == 0 ? g : g - hq;
            const bf16 *bias = (kind == 0 ? p.q_bias : p.k_bias) + hh * HD;
            // rotated in place: element i reads x1[i], x2[i] before writing them
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                float b1[8], b2[8];
                {
                    const uint4 u1 = reinterpret_cast<const uint4 *>(bias + d0)[v];
                    const uint4 u2 = reinterpret_cast<const uint4 *>(bias + kHalf + d0)[v];
                    const __nv_bfloat162 *h1 = reinterpret_cast<const __nv_bfloat162 *>(&u1);
                    const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&u2);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        b1[2 * i] = __low2float(h1[i]);
                        b1[2 * i + 1] = __high2float(h1[i]);
                        b2[2 * i] = __low2float(h2[i]);
                        b2[2 * i + 1] = __high2float(h2[i]);
                    }
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int i = 8 * v + e;
                    const float v1 = __fadd_rn(x1[i], b1[e]), v2 = __fadd_rn(x2[i], b2[e]);
                    x1[i] = rot_sub(v1, w.cs[i], v2, w.sn[i]);
                    x2[i] = rot_add(v1, w.sn[i], v2, w.cs[i]);
                }
            }
        }
        // The row: q / k rotated, v (and rows rope_append skips) as projected.
        o.begin();
        o.put(row, live, hc + d0, 0, x1);
        o.put(row, live, hc + kHalf + d0, 1, x2);
        if (appendable) {
            if (kind == 1 && w.rope_ok) {
                bf16 *dst = p.k_pool + base + (g - hq) * stride_blk;
                store32(dst + d0, x1);
                store32(dst + kHalf + d0, x2);
            } else if (kind == 2) {  // past the RoPE table k is not appended, v still is
                const int vh = g - hq - hkv;
                const bf16 *vb = p.v_bias + vh * HD;
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const uint4 u1 = reinterpret_cast<const uint4 *>(vb + d0)[v];
                    const uint4 u2 = reinterpret_cast<const uint4 *>(vb + kHalf + d0)[v];
                    const __nv_bfloat162 *h1 = reinterpret_cast<const __nv_bfloat162 *>(&u1);
                    const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&u2);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        x1[8 * v + 2 * i] = __fadd_rn(x1[8 * v + 2 * i], __low2float(h1[i]));
                        x1[8 * v + 2 * i + 1] = __fadd_rn(x1[8 * v + 2 * i + 1], __high2float(h1[i]));
                        x2[8 * v + 2 * i] = __fadd_rn(x2[8 * v + 2 * i], __low2float(h2[i]));
                        x2[8 * v + 2 * i + 1] = __fadd_rn(x2[8 * v + 2 * i + 1], __high2float(h2[i]));
                    }
                }
                bf16 *dst = p.v_pool + base + vh * stride_blk;
                store32(dst + d0, x1);
                store32(dst + kHalf + d0, x2);
            }
        }
        o.issue(2, hc + d0, hc + kHalf + d0, y, y < p.M);
    }
}

// ------------------------------------------------------------ CTA pairs --
// The same GEMM over 256 x 256 tiles shared by a cluster of two CTAs
// (tcgen05.mma.cta_group::2): CTA r loads rows [128 r, 128 r + 128) of the
// tile's x rows and of its w rows, so a K block costs each CTA 32 KiB of
// loads instead of 48 KiB. Rank 0 issues the MMAs; the pair's loads complete
// on its stage barriers, its commits arrive on both CTAs' barriers, and both
// CTAs' epilogue warps release the accumulator to it. The epilogue writes its
// rows through shared memory with TMA stores (OutStaged).
constexpr int kStages2 = 5;
constexpr uint32_t kHalfTile = 128 * kBK * 2;  // 16 KiB: 128 rows of one operand
constexpr uint32_t kStageBytes2 = 2 * kHalfTile;
constexpr uint32_t kStageOut = 8192;  // per epilogue warp: 2 buffers x 2 boxes of 32 x 32
constexpr int kSmem2 = kStages2 * kStageBytes2 + kEpiWarps * kStageOut + 1024;
constexpr uint32_t kIdesc2 = idesc_bf16_f32(256, kBN, 0);
constexpr int kBM2 = 256;

template <int EPI, int HD>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsG, 1)
    proj_gemm2_kernel(const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_out, const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *gen = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[kStages2];
    __shared__ __align__(8) uint64_t empty[kStages2];
    __shared__ __align__(8) uint64_t acc_full[2];
    __shared__ __align__(8) uint64_t acc_empty[2];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages2; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * kEpiWarps);
        }
        s_abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_2sm(&tmem_base_sh, kTmemColsG);
        tmem_relinquish_2sm();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers exist and the pair's TMEM is allocated
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    const int pairs = (int)(gridDim.x >> 1), pair = (int)(blockIdx.x >> 1);
    const int tiles = p.m_tiles * p.n_tiles;
    const int kblocks = (p.K + kBK - 1) / kBK;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA --
        if (lane == 0) {
            prefetch_tensormap(&tm_a);
            prefetch_tensormap(&tm_b);
            int it = 0;
            bool ok = true;
            for (int tile = pair; tile < tiles && ok; tile += pairs) {
                const int mt = tile / p.n_tiles, nt = tile - mt * p.n_tiles;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kStages2;
                    if (it >= kStages2 &&
                        !mbar_wait_bounded_cluster(&empty[s], ((it / kStages2) - 1) & 1, &s_abort,
                                                   p.status)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * kStageBytes2);
                    const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
                    uint8_t *st = gen + s * kStageBytes2;
                    tma_load_2d_2sm(st, &tm_a, kb * kBK, mt * kBM2 + (int)rank * 128, fb);
                    tma_load_2d_2sm(st + kHalfTile, &tm_b, kb * kBK, nt * kBN + (int)rank * 128, fb);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------- MMA (rank 0 only) --
        if (leader && lane == 0) {
            int it = 0, tl = 0;
            bool ok = true;
            for (int tile = pair; tile < tiles && ok; tile += pairs, ++tl) {
                const int buf = tl & 1;
                if (tl >= 2 && !mbar_wait_bounded_cluster(&acc_empty[buf], ((tl >> 1) - 1) & 1,
                                                          &s_abort, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + buf * kBN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kStages2;
                    if (!mbar_wait_bounded_cluster(&full[s], (it / kStages2) & 1, &s_abort,
                                                   p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(gen + s * kStageBytes2), b = a + kHalfTile;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_bf16_2sm(d, sw128_desc(a + kk * 32, 16, 1024),
                                      sw128_desc(b + kk * 32, 16, 1024), kIdesc2,
                                      (kb > 0 || kk > 0) ? 1u : 0u);
                    umma_commit_2sm(&empty[s], 0x3);  // frees the stage in both CTAs
                }
                if (ok) umma_commit_2sm(&acc_full[buf], 0x3);
            }
        }
    } else {
        // ----------------------------------------------------------- epilogue --
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const uint32_t release = mapa_shared(smem_u32(&acc_empty[0]), 0);
        OutStaged o{gen + kStages2 * kStageBytes2 + (warp - 2) * kStageOut, &tm_out, 0, lane};
        if (lane == 0) prefetch_tensormap(&tm_out);
        int tl = 0;
        for (int tile = pair; tile < tiles; tile += pairs, ++tl) {
            const int buf = tl & 1;
            const int mt = tile / p.n_tiles, nt = tile - mt * p.n_tiles;
            const int row = mt * kBM2 + (int)rank * 128 + r, col0 = nt * kBN;
            const uint32_t tacc = tmem + ((uint32_t)(quad * 32) << 16) + buf * kBN;
            const int y = mt * kBM2 + (int)rank * 128 + quad * 32;
            if constexpr (EPI == kQkvRope) {
                QkvRow<HD> w;
                w.load(p, row, col0, half);  // overlaps the tile's MMAs
                if (!mbar_wait_bounded_cluster(&acc_full[buf], (tl >> 1) & 1, &s_abort, p.status))
                    break;
                tc_fence_after();
                epilogue_qkv<HD>(p, tacc, row, y, col0, half, w, o);
            } else {
                if (!mbar_wait_bounded_cluster(&acc_full[buf], (tl >> 1) & 1, &s_abort, p.status))
                    break;
                tc_fence_after();
                epilogue_rows<EPI>(p, tacc, row, y, col0, half, o);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(release + buf * 8);  // acc_empty[buf] of rank 0
        }
        o.drain();
    }
    tc_fence_before();
    cluster_sync();  // the pair's MMAs, copies and arrivals are over before TMEM is freed
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_2sm(tmem, kTmemColsG);
    }
}

// Clusters of two that fit on the current device at once (cached per device).
template <int EPI, int HD>
int pair_slots() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return sm_count() / 2;
    }
    if (!cached[dev]) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(kThreadsG);
        cfg.dynamicSmemBytes = kSmem2;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, proj_gemm2_kernel<EPI, HD>, &cfg) != cudaSuccess ||
            n < 1) {
            cudaGetLastError();
            n = sm_count() / 2;
        }
        cached[dev] = n;
    }
    return cached[dev];
}

// M > 128: tiles of 256 rows on CTA pairs; the pair count is what fits at once.
template <int EPI, int HD>
int launch_gemm2(GemmParams prm, const void *x, int64_t x_stride, const void *w,
                 int64_t w_stride, cudaStream_t stream) {
    prm.m_tiles = (prm.M + kBM2 - 1) / kBM2;
    CUtensorMap ma, mb, mo;
    int rc = tensor_map_2d_sw128(x, prm.K, prm.M, x_stride * 2, kBK, 128, &ma);
    if (rc) return rc;
    rc = tensor_map_2d_sw128(w, prm.K, prm.N, w_stride * 2, kBK, 128, &mb);
    if (rc) return rc;
    rc = tensor_map_2d(prm.out, prm.N, prm.M, prm.out_stride * 2, 32, 32, 64, &mo);
    if (rc) return rc;
    rc = ensure_smem_attr((const void *)proj_gemm2_kernel<EPI, HD>, kSmem2);
    if (rc) return rc;
    const int tiles = prm.m_tiles * prm.n_tiles;
    const int slots = pair_slots<EPI, HD>();
    const int pairs = tiles < slots ? tiles : slots;
    proj_gemm2_kernel<EPI, HD><<<2 * pairs, kThreadsG, kSmem2, stream>>>(ma, mb, mo, prm);
    return launch_status();
}

// M <= 128 token rows (a decode step): the weight-streaming kernel of
// proj_decode.cu; more rows: 256 x 256 tiles on CTA pairs.
template <int EPI, int HD>
int launch_any(const GemmParams &prm, const void *x, int64_t x_stride, const void *w,
               int64_t w_stride, cudaStream_t stream) {
    if (prm.M > kDecodeProjMaxRows) return launch_gemm2<EPI, HD>(prm, x, x_stride, w, w_stride, stream);
    DecodeProjArgs a{};
    a.epi = EPI;  // kPlain / kResidual / kQkvRope: the decode kernel's numbering
    a.M = prm.M;
    a.N = prm.N;
    a.K = prm.K;
    a.out = prm.out;
    a.out_stride = prm.out_stride;
    a.x = x;
    a.x_stride = x_stride;
    a.w = w;
    a.w_stride = w_stride;
    a.residual = prm.residual;
    a.res_stride = prm.res_stride;
    a.tokens_per_seq = prm.tokens_per_seq;
    a.positions = prm.positions;
    a.q_bias = prm.q_bias;
    a.k_bias = prm.k_bias;
    a.v_bias = prm.v_bias;
    a.cos_t = prm.cos_t;
    a.sin_t = prm.sin_t;
    a.rope_rows = prm.rope_rows;
    a.k_pool = prm.k_pool;
    a.v_pool = prm.v_pool;
    a.num_blocks = prm.num_blocks;
    a.num_layers = prm.num_layers;
    a.layer = prm.layer;
    a.num_q_heads = prm.num_q_heads;
    a.num_kv_heads = prm.num_kv_heads;
    a.head_dim = prm.head_dim;
    a.tables = prm.tables;
    a.table_stride = prm.table_stride;
    a.status = prm.status;
    return decode_proj_launch(a, stream);
}

int check_gemm_shape(const void *out, int64_t out_stride, const void *x, int64_t x_stride,
                     const void *w, int64_t w_stride, int M, int N, int K) {
    if (!out || !x || !w) return LC_ERR_INVALID_ARGUMENT;
    if (M < 0 || N <= 0 || K <= 0 || (N & 31) || (K & 7)) return LC_ERR_UNSUPPORTED_SHAPE;
    if (x_stride < K || w_stride < K || out_stride < N) return LC_ERR_INVALID_ARGUMENT;
    if (!aligned16(out) || !aligned16(x) || !aligned16(w) || (x_stride & 7) || (w_stride & 7) ||
        (out_stride & 7))
        return LC_ERR_MISALIGNED;
    if ((int64_t)M >= (int64_t(1) << 31) - kBM || (int64_t)N >= (int64_t(1) << 31) - kBN)
        return LC_ERR_INVALID_ARGUMENT;
    return LC_OK;
}

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" int lc_proj_gemm(void *out, int64_t out_stride, const void *x, int64_t x_stride,
                            const void *w, int64_t w_stride, int M, int N, int K,
                            const void *residual, int64_t res_stride, lc_stream_t stream) {
    int rc = check_gemm_shape(out, out_stride, x, x_stride, w, w_stride, M, N, K);
    if (rc) return rc;
    if (residual && (!aligned16(residual) || (res_stride & 7))) return LC_ERR_MISALIGNED;
    if (residual && res_stride < N) return LC_ERR_INVALID_ARGUMENT;
    if (M == 0) return LC_OK;
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.m_tiles = (M + kBM - 1) / kBM;
    p.n_tiles = (N + kBN - 1) / kBN;
    p.out = (bf16 *)out;
    p.out_stride = out_stride;
    p.residual = (const bf16 *)residual;
    p.res_stride = res_stride;
    cudaStream_t s = as_stream(stream);
    return residual ? launch_any<kResidual, 64>(p, x, x_stride, w, w_stride, s)
                    : launch_any<kPlain, 64>(p, x, x_stride, w, w_stride, s);
}

extern "C" int lc_qkv_proj_rope_append(void *qkv, int64_t row_stride, const void *x,
                                       int64_t x_stride, const void *w_qkv, int64_t w_stride,
                                       int hidden, int num_seqs, int tokens_per_seq,
                                       const int *positions, const void *q_bias,
                                       const void *k_bias, const void *v_bias,
                                       const float *cos_cache, const float *sin_cache,
                                       int rope_rows, void *k_pool, void *v_pool,
                                       int64_t num_blocks, int num_layers, int layer,
                                       int num_q_heads, int num_kv_heads, int head_dim,
                                       const int *block_tables, int table_stride,
                                       int *dev_status, lc_stream_t stream) {
    if (!positions || !q_bias || !k_bias || !v_bias || !cos_cache || !sin_cache || !k_pool ||
        !v_pool || !block_tables)
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (num_seqs < 0 || tokens_per_seq <= 0 || num_layers <= 0 || layer < 0 ||
        layer >= num_layers || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
        table_stride <= 0 || rope_rows <= 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if ((int64_t)num_seqs * tokens_per_seq >= (int64_t(1) << 31) - kBM)
        return LC_ERR_INVALID_ARGUMENT;
    const int M = num_seqs * tokens_per_seq;
    const int N = (num_q_heads + 2 * num_kv_heads) * head_dim;
    int rc = check_gemm_shape(qkv, row_stride, x, x_stride, w_qkv, w_stride, M, N, hidden);
    if (rc) return rc;
    if (!aligned16(q_bias) || !aligned16(k_bias) || !aligned16(v_bias) || !aligned16(cos_cache) ||
        !aligned16(sin_cache) || !aligned16(k_pool) || !aligned16(v_pool))
        return LC_ERR_MISALIGNED;
    if (M == 0) return LC_OK;
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = hidden;
    p.m_tiles = (M + kBM - 1) / kBM;
    p.n_tiles = (N + kBN - 1) / kBN;
    p.out = (bf16 *)qkv;
    p.out_stride = row_stride;
    p.tokens_per_seq = tokens_per_seq;
    p.positions = positions;
    p.q_bias = (const bf16 *)q_bias;
    p.k_bias = (const bf16 *)k_bias;
    p.v_bias = (const bf16 *)v_bias;
    p.cos_t = cos_cache;
    p.sin_t = sin_cache;
    p.rope_rows = rope_rows;
    p.k_pool = (bf16 *)k_pool;
    p.v_pool = (bf16 *)v_pool;
    p.num_blocks = num_blocks;
    p.num_layers = num_layers;
    p.layer = layer;
    p.num_q_heads = num_q_heads;
    p.num_kv_heads = num_kv_heads;
    p.head_dim = head_dim;
    p.tables = block_tables;
    p.table_stride = table_stride;
    p.status = dev_status;
    cudaStream_t s = as_stream(stream);
    return head_dim == 64 ? launch_any<kQkvRope, 64>(p, x, x_stride, w_qkv, w_stride, s)
                          : launch_any<kQkvRope, 128>(p, x, x_stride, w_qkv, w_stride, s);
}
