// proj_decode.cu - the projections either side of attention for a decode
// step: out[M][N] = x[M][K] . w[N][K]^T with M <= 128 token rows (one row per
// sequence of the batch), as Qwen2Model::matmul_bf16 computes them per token
// (src/models.rs:252-292: cublasGemmEx, CUBLAS_COMPUTE_32F, bf16 C; qkv_proj at
// :470-483, o_proj with beta 1 at :553-566). At this size the GEMM is bound by
// reading the weights once (x is a few hundred KiB and stays in L2), so the
// kernel is laid out to stream w over as many SMs as possible:
//
//  * The MMA's M dimension is the weights: a tile is 64 weight rows (output
//    columns) in two boxes of 32, the first holding dims d and the second
//    dims d + head_dim/2 of the same head at head_dim 128 (the pairs RoPE
//    rotates together; at head_dim 64 a tile is one head); the token rows are
//    the MMA's N (padded to a multiple of 16). tcgen05.mma M64 x N(tokens) x
//    K16, bf16 in, fp32 accumulate in TMEM, where weight row m of the tile
//    sits in lane (m % 16) + 32 (m / 16).
//  * A cluster of `split` CTAs (a power of two up to 8) shares one tile, CTA r
//    taking the r-th slice of K: tiles x split CTAs cover the SMs (one CTA per
//    SM; the split is the widest whose clusters all fit at once).
//  * Warps 2-9 stream the CTA's K slice into a 192 KiB ring with cp.async,
//    four K blocks per ring slot, so that one warp instruction fetches 512
//    contiguous bytes of one weight row (TMA boxes of 32 rows x 128 bytes from
//    rows 7 KiB apart ran at ~27 GB/s per SM: the copy engine handled them one
//    128-byte row at a time, arrivals 0.45 us apart per stage); the copies
//    land in the 128-byte-swizzled layout the MMA reads. The weight loads of
//    the first slots are issued before the programmatic-dependency wait, the
//    token rows (written by the preceding kernel) after it. Warp 1 issues the
//    MMAs. Then warps 2-9 move the CTA's partial tile from TMEM into its
//    shared memory (the idle ring).
//  * Cluster reduction over distributed shared memory: CTA r owns 32/split of
//    the tile's 32 row pairs and sums them over the cluster's partials in rank
//    order (the same order whatever the timing), then runs the epilogue on
//    them.
//
// Epilogues (the arithmetic of proj_gemm.cu, element by element):
//   plain     out = bf16(acc)
//   residual  out = bf16(acc + residual)        (residual may be out itself)
//   qkv rope  the QKV projection followed by what lc_rope_append does to its
//             rows: rounded to bf16, bias added, q and k rotated and stored
//             back, k appended rotated and v + bias appended to the pools.
//
// Every mbarrier wait is bounded (LC_DEV_TIMEOUT); every thread reaches both
// cluster barriers on every path, so a CTA that gave up still releases the
// others.
#include <climits>

#include "lc_common.cuh"
#include "lc_host.h"
#include "lc_tcgen05.cuh"
#include "rope_math.cuh"

namespace lc {
namespace {

constexpr int kPRows = 64;    // weight rows per tile (the MMA's M)
constexpr int kPK = 64;       // K per stage: one 128-byte swizzle row
constexpr int kPMaxStages = 16;
constexpr uint32_t kPRingBytes = 192 * 1024;
constexpr int kPLoadWarps = 8;  // copy, then stage and finish the tile
constexpr int kPThreads = 64 + 32 * kPLoadWarps;  // idle warp, MMA warp, loading warps
constexpr int kPPairs = kPRows / 2;
constexpr uint32_t kPWTile = kPRows * kPK * 2;         // 8 KiB: two boxes of 32 rows
constexpr int kPGroupKB = 4;  // K blocks per ring slot: 512 contiguous bytes of a row
constexpr int kPSmem = kPRingBytes + 1024;  // + 1024-byte alignment slack
constexpr int kPMaxSplit = 8;
constexpr uint32_t kPTmemCols = 128;
// Cluster sums of the items a CTA finishes (<= 128 token rows x 32 row pairs
// float2 = 32 KiB), in the ring past the staged tile (<= 64 x 132 fp32).
constexpr uint32_t kPSumsOff = 64 * 1024;
constexpr int kPBatch = 4;  // items whose partials are loaded together
static_assert(kPSumsOff + kDecodeProjMaxRows * 32 * 8 <= kPRingBytes, "sums fit the ring");

enum DecEpilogue { kDecPlain = 0, kDecResidual = 1, kDecQkv = 2 };

struct DecProjParams {
    int M, N, K;
    const bf16 *w, *x;
    int64_t w_stride, x_stride;
    int Mt;       // token rows padded to a multiple of 16 (the MMA's N)
    int split;    // CTAs per cluster (K slices)
    int stages;   // ring slots: groups of kPGroupKB (w tile + x tile) stages
    uint32_t stage_bytes;  // one K block: w tile (8 KiB) + x tile
    int kblocks;  // K / 64, rounded up
    int pdl_mode;
    bf16 *out;
    int64_t out_stride;
    const bf16 *residual;
    int64_t res_stride;
    // qkv rope: token rows (row / tokens_per_seq = sequence), columns
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

// Staged partial tile: [64 weight rows][Mt + 4] fp32 (the padding spreads the
// rows over the shared-memory banks).
__host__ __device__ __forceinline__ int stage_pitch(int Mt) { return Mt + 4; }

// First weight rows of the two 32-row boxes of tile t. With heads of 128 dims
// (QKV) box 1 holds the partners (dim + 64) of box 0's dims; otherwise the
// boxes are the tile's 64 consecutive rows (at head_dim 64 exactly one head:
// dim d in box 0, its partner d + 32 in box 1). Tile-local row pair p (< 32)
// is rows (r0 + p, r1 + p).
__host__ __device__ __forceinline__ void tile_rows(int t, bool heads128, int &r0, int &r1) {
    if (heads128) {
        r0 = (t >> 1) * 128 + (t & 1) * 32;
        r1 = r0 + 64;
    } else {
        r0 = t * 64;
        r1 = r0 + 32;
    }
}

// 16-byte asynchronous copy global -> shared (zero fill when !valid).
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
// The mbarrier counts this thread's arrival once all its earlier cp.async copies
// have landed (no separate arrive).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// bf16(acc) back as a float: the value the reference's qkv buffer holds.
__device__ __forceinline__ float round_bf16_dec(float x) {
    return __bfloat162float(__float2bfloat16(x));
}

// Pool offset of (position, kv head 0) for token row `row`, or -1 when it must
// not be appended (status bits set), as rope_append.cu does.
__device__ __forceinline__ int64_t dec_pool_base(const DecProjParams &p, int row, int pos) {
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

// Plain / residual epilogue of one output element (token row m, column col).
template <int EPI>
__device__ __forceinline__ void dec_store_plain(const DecProjParams &p, int m, int col, float acc) {
    if (col >= p.N) return;
    float f = acc;
    if constexpr (EPI == kDecResidual)
        f = __fadd_rn(acc, __bfloat162float(p.residual[(int64_t)m * p.res_stride + col]));
    p.out[(int64_t)m * p.out_stride + col] = __float2bfloat16(f);
}

// QKV epilogue of one row pair (token row m, columns col and col + HD/2 of
// one head): what epilogue_qkv in proj_gemm.cu does per element, i.e.
// rope_append_vec_kernel's arithmetic on the bf16-rounded projection. The row
// keeps the projection where rope_append leaves it (v, a negative position, a
// position past the RoPE table).
template <int HD>
__device__ __forceinline__ void dec_store_qkv(const DecProjParams &p, int m, int col, float acc_a,
                                              float acc_b) {
    constexpr int kHalf = HD / 2;
    if (col >= p.N) return;
    const int hq = p.num_q_heads, hkv = p.num_kv_heads;
    const int g = col / HD, d = col - g * HD;  // head over [q | k | v], dim < HD/2
    const int kind = g < hq ? 0 : (g < hq + hkv ? 1 : 2);
    const int pos = p.positions[m];
    if (pos < 0 || pos >= p.rope_rows) set_status(p.status, LC_DEV_BAD_POS);
    const bool rope_ok = pos >= 0 && pos < p.rope_rows;
    float x1 = round_bf16_dec(acc_a), x2 = round_bf16_dec(acc_b);
    const int64_t base = pos >= 0 && kind != 0 ? dec_pool_base(p, m, pos) : -1;
    if (pos >= 0 && kind != 2 && rope_ok) {
        const int hh = kind == 0 ? g : g - hq;
        const bf16 *bias = (kind == 0 ? p.q_bias : p.k_bias) + hh * HD;
        const float c = p.cos_t[(int64_t)pos * kHalf + d], s = p.sin_t[(int64_t)pos * kHalf + d];
        const float v1 = __fadd_rn(x1, __bfloat162float(bias[d]));
        const float v2 = __fadd_rn(x2, __bfloat162float(bias[d + kHalf]));
        x1 = rot_sub(v1, c, v2, s);
        x2 = rot_add(v1, s, v2, c);
    }
    bf16 *orow = p.out + (int64_t)m * p.out_stride;
    orow[col] = __float2bfloat16(x1);
    orow[col + kHalf] = __float2bfloat16(x2);
    if (pos >= 0 && base >= 0) {
        const int64_t stride_blk = (int64_t)kBlockSize * HD;
        if (kind == 1 && rope_ok) {  // past the RoPE table k is not appended, v still is
            bf16 *dst = p.k_pool + base + (g - hq) * stride_blk;
            dst[d] = __float2bfloat16(x1);
            dst[d + kHalf] = __float2bfloat16(x2);
        } else if (kind == 2) {
            const int vh = g - hq - hkv;
            const bf16 *vb = p.v_bias + vh * HD;
            bf16 *dst = p.v_pool + base + vh * stride_blk;
            dst[d] = __float2bfloat16(__fadd_rn(x1, __bfloat162float(vb[d])));
            dst[d + kHalf] = __float2bfloat16(__fadd_rn(x2, __bfloat162float(vb[d + kHalf])));
        }
    }
}

template <int EPI, int HD>
__global__ void __launch_bounds__(kPThreads, 1)
    proj_decode_kernel(const DecProjParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *gen = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[kPMaxStages];
    __shared__ __align__(8) uint64_t empty[kPMaxStages];
    __shared__ __align__(8) uint64_t acc_full;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = (int)cluster_ctarank();
    const int tile = (int)blockIdx.x / p.split;
    int wr0, wr1;
    tile_rows(tile, EPI == kDecQkv && HD == 128, wr0, wr1);
    const int kb0 = rank * p.kblocks / p.split, kb1 = (rank + 1) * p.kblocks / p.split;
    const int nkb = kb1 - kb0;
    const int ngroups = (nkb + kPGroupKB - 1) / kPGroupKB;
    const uint32_t group_bytes = kPGroupKB * p.stage_bytes;
    const uint32_t idesc = idesc_bf16_f32(kPRows, p.Mt, 0);

    griddep_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 32 * kPLoadWarps);  // the loading warps' cp.async arrivals
            mbar_init(&empty[s], 1);
        }
        mbar_init(&acc_full, 1);
        s_abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_sh, kPTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp == 1) {
        // ---------------------------------------------------------------- MMA --
        if (lane == 0) {
            bool ok = true;
            for (int gi = 0; gi < ngroups; ++gi) {
                const int s = gi % p.stages;
                if (!mbar_wait_bounded(&full[s], (gi / p.stages) & 1, &s_abort, p.status)) {
                    ok = false;
                    break;
                }
                // The copies are generic-proxy writes; the MMAs read through the
                // async proxy.
                fence_proxy_async_smem();
                tc_fence_after();
                const int nj = min(kPGroupKB, nkb - gi * kPGroupKB);
                for (int j = 0; j < nj; ++j) {
                    const uint32_t a = smem_u32(gen + s * group_bytes + j * p.stage_bytes);
                    const uint32_t b = a + kPWTile;
#pragma unroll
                    for (int kk = 0; kk < kPK / 16; ++kk)
                        umma_bf16(tmem, sw128_desc(a + kk * 32, 16, 1024),
                                  sw128_desc(b + kk * 32, 16, 1024), idesc,
                                  (gi > 0 || j > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&empty[s]);  // the group's slot is free once these MMAs are done
            }
            if (ok && nkb > 0) umma_commit(&acc_full);
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------ loads (cp.async) --
        // Warps 2-9 copy each group of kPGroupKB K blocks: one warp instruction
        // moves 512 contiguous bytes of one weight (or token) row, lane l taking
        // K block l / 8, 16-byte chunk l % 8, into the 128-byte-swizzled tile
        // the MMA reads (chunk c of row r at r * 128 + ((c ^ (r % 8)) * 16)).
        // Rows past N or M and K past the end are zero-filled. The first
        // groups' weights are requested before the programmatic-dependency
        // wait, the token rows after it.
        // Each thread's rows, their source rows and swizzled offsets are fixed
        // for the whole K slice: computed once, so that a group is a run of
        // independent copies (one loading warp per SM sub-partition cannot
        // hide a chain of address arithmetic per copy).
        const int pw = warp - 2;
        const int jl = lane >> 3, cl = lane & 7;
        constexpr int kWRows = kPRows / kPLoadWarps;  // weight rows per thread
        constexpr int kXRows = kDecodeProjMaxRows / kPLoadWarps;
        const bf16 *wsrc[kWRows];
        uint32_t wdst[kWRows];
        bool wok[kWRows];
#pragma unroll
        for (int i = 0; i < kWRows; ++i) {
            const int r = pw + kPLoadWarps * i;
            const int grow = r < 32 ? wr0 + r : wr1 + (r - 32);
            wok[i] = grow < p.N;
            wsrc[i] = p.w + (wok[i] ? (int64_t)grow * p.w_stride + cl * 8 : 0);
            wdst[i] = (uint32_t)(r * 128 + ((cl ^ (r & 7)) << 4));
        }
        const bf16 *xsrc = p.x + (int64_t)pw * p.x_stride + cl * 8;
        const int64_t xstep = (int64_t)kPLoadWarps * p.x_stride;
        auto load_w = [&](int slot, int gi) {
            uint8_t *base = gen + slot * group_bytes + jl * p.stage_bytes;
            const int kb = kb0 + gi * kPGroupKB + jl;
            const bool kok = kb < kb1 && kb * kPK + cl * 8 < p.K;
            const int64_t ko = kok ? (int64_t)kb * kPK : 0;
#pragma unroll
            for (int i = 0; i < kWRows; ++i)
                cp_async16(base + wdst[i], kok && wok[i] ? wsrc[i] + ko : p.w, kok && wok[i]);
        };
        auto load_x = [&](int slot, int gi) {
            uint8_t *base = gen + slot * group_bytes + jl * p.stage_bytes + kPWTile;
            const int kb = kb0 + gi * kPGroupKB + jl;
            const bool kok = kb < kb1 && kb * kPK + cl * 8 < p.K;
            const int64_t ko = kok ? (int64_t)kb * kPK : 0;
#pragma unroll
            for (int i = 0; i < kXRows; ++i) {
                const int t = pw + kPLoadWarps * i;
                if (t < p.Mt) {
                    const bool ok = kok && t < p.M;
                    cp_async16(base + t * 128 + ((cl ^ (t & 7)) << 4),
                               ok ? xsrc + i * xstep + ko : p.x, ok);
                }
            }
        };
        const int pre = min(ngroups, p.stages);
        for (int gi = 0; gi < pre; ++gi) load_w(gi, gi);
        if (p.pdl_mode) griddep_wait();
        for (int gi = 0; gi < pre; ++gi) {
            load_x(gi, gi);
            cp_async_arrive_noinc(&full[gi]);  // lands with this thread's copies so far
        }
        int slot = 0;
        uint32_t wrap_phase = 0;  // parity of the slot's previous use
        for (int gi = pre; gi < ngroups; ++gi) {
            if (!mbar_wait_bounded(&empty[slot], wrap_phase, &s_abort, p.status)) break;
            load_w(slot, gi);
            load_x(slot, gi);
            cp_async_arrive_noinc(&full[slot]);
            if (++slot == p.stages) {
                slot = 0;
                wrap_phase ^= 1u;
            }
        }
        cp_async_wait_all();  // no copy may land in the ring after this point

        // ------------------------------- partial tile: TMEM -> shared memory --
        // The ring is idle once the accumulator is complete (every stage's
        // MMAs have read it); it holds the staged tile [64][Mt + 4] fp32.
        // An M64 accumulator fills lanes 0-15 of each 32-lane quadrant: lane i
        // of quadrant q holds the tile's weight row 16 q + i.
        const int quad = warp & 3;
        const int row = quad * 16 + lane;
        float *stg = reinterpret_cast<float *>(gen);
        const int pitch = stage_pitch(p.Mt);
        bool have = nkb > 0 && mbar_wait_bounded(&acc_full, 0, &s_abort, p.status);
        have = __all_sync(0xffffffffu, have);
        tc_fence_after();
        // warps 2-5 move columns [0, 32), [64, 96), ...; warps 6-9 the others
        for (int c0 = 32 * (pw >> 2); c0 < p.Mt; c0 += 64) {
            uint32_t r[32];
            if (have) {
                tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c0, r);
                tmem_wait_ld_regs(r);
            }
            if (lane < 16) {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (c0 + i < p.Mt) stg[row * pitch + c0 + i] = have ? __uint_as_float(r[i]) : 0.f;
            }
        }
    }
    // Every CTA's staged tile is complete and visible to the cluster.
    tc_fence_before();
    __syncwarp();
    cluster_sync();

    // ------------------------------------------- reduction over the cluster --
    // Each epilogue thread takes a contiguous run of (token row, row pair)
    // items, all of one token row where the run allows, so that the row's
    // position and block-table entry are read once. First the sums of all its
    // items over the cluster's partials (rank order: the same sum whatever the
    // timing), with every distributed-shared-memory load of a batch in flight
    // at once, into this CTA's own shared memory past the staged tile; then
    // the CTA tells the cluster it is done reading, and the epilogue runs
    // while the slower CTAs finish theirs.
    const bool run = warp >= 2 && !s_abort;
    const int npr = kPPairs / p.split;  // row pairs this CTA finishes (a power of two)
    const int lnpr = 5 - (__ffs(p.split) - 1);
    const int items = p.M * npr;
    constexpr int kET = 32 * kPLoadWarps;     // epilogue threads
    const int ipt = (items + kET - 1) / kET;  // items per epilogue thread
    const int it0 = (threadIdx.x - 64) * ipt;
    const int it1 = min(items, it0 + ipt);
    float2 *sums = reinterpret_cast<float2 *>(gen + kPSumsOff);
    if (run) {
        const int pr0 = rank * npr;
        const int pitch = stage_pitch(p.Mt);
        const uint32_t stg = smem_u32(gen);
        uint32_t peer[kPMaxSplit];
#pragma unroll
        for (int r = 0; r < kPMaxSplit; ++r) peer[r] = r < p.split ? mapa_shared(stg, r) : 0u;
        for (int i0 = it0; i0 < it1; i0 += kPBatch) {
            float va[kPBatch][kPMaxSplit], vb[kPBatch][kPMaxSplit];
#pragma unroll
            for (int u = 0; u < kPBatch; ++u) {
                const int item = i0 + u;
                const int m = item >> lnpr, ra = pr0 + (item & (npr - 1)), rb = ra + 32;
#pragma unroll
                for (int r = 0; r < kPMaxSplit; ++r) {
                    if (item < it1 && r < p.split) {
                        va[u][r] = ld_dsmem_f32(peer[r] + (uint32_t)(ra * pitch + m) * 4u);
                        vb[u][r] = ld_dsmem_f32(peer[r] + (uint32_t)(rb * pitch + m) * 4u);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kPBatch; ++u) {
                float a = 0.f, b = 0.f;
#pragma unroll
                for (int r = 0; r < kPMaxSplit; ++r) {
                    if (r < p.split) {
                        a += va[u][r];
                        b += vb[u][r];
                    }
                }
                if (i0 + u < it1) sums[i0 + u] = make_float2(a, b);
            }
        }
    }
    // This CTA no longer reads the others' staged tiles.
    __syncwarp();
    cluster_arrive();

    if (run) {
        // --------------------------------------------------------- epilogue --
        if (p.pdl_mode) griddep_wait();  // outputs / pools after the preceding kernel
        const int pr0 = rank * npr;
        for (int item = it0; item < it1; ++item) {
            const int m = item >> lnpr, ra = pr0 + (item & (npr - 1));  // tile-local rows ra, ra + 32
            const float2 ab = sums[item];
            const int col = wr0 + ra, colb = wr1 + ra;  // colb = col + head_dim/2 (QKV)
            if constexpr (EPI == kDecQkv) {
                dec_store_qkv<HD>(p, m, col, ab.x, ab.y);
            } else {
                dec_store_plain<EPI>(p, m, col, ab.x);
                dec_store_plain<EPI>(p, m, colb, ab.y);
            }
        }
    }
    // No CTA leaves while another may still read its staged tile.
    __syncwarp();
    cluster_wait();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kPTmemCols);
    }
}

// Clusters of `split` CTAs (one CTA per SM: the ring takes most of shared
// memory) that the device runs at once, per split; cached per device.
// Shared-memory size and carveout of the kernel (once per instance and device).
template <int EPI, int HD>
int prepare_kernel() {
    static bool done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    int rc = ensure_smem_attr((const void *)proj_decode_kernel<EPI, HD>, kPSmem);
    if (rc) return rc;
    if (!done[dev]) {
        if (cudaFuncSetAttribute(proj_decode_kernel<EPI, HD>,
                                 cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
            cudaGetLastError();
            return LC_ERR_CUDA;
        }
        done[dev] = true;
    }
    return LC_OK;
}

template <int EPI, int HD>
int ctas_per_sm() {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, proj_decode_kernel<EPI, HD>, kPThreads,
                                                      kPSmem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

template <int EPI, int HD>
int max_clusters(int split) {
    static int cached[64][4] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 0;
    }
    const int idx = split == 1 ? 0 : split == 2 ? 1 : split == 4 ? 2 : 3;
    if (!cached[dev][idx]) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(split);
        cfg.blockDim = dim3(kPThreads);
        cfg.dynamicSmemBytes = kPSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = split;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, proj_decode_kernel<EPI, HD>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        cached[dev][idx] = n > 0 ? n : -1;
    }
    return cached[dev][idx] > 0 ? cached[dev][idx] : 0;
}

// The widest K split (a power of two, at most 8 and at most the number of
// 64-wide K blocks) whose clusters all fit on the device at once.
template <int EPI, int HD>
int choose_split(int n_tiles, int kblocks) {
    for (int s = kPMaxSplit; s > 1; s >>= 1) {
        if (s > kblocks) continue;
        if (max_clusters<EPI, HD>(s) >= n_tiles) return s;
    }
    return 1;
}

template <int EPI, int HD>
int launch_decode_proj(DecProjParams prm, const void *x, int64_t x_stride, const void *w,
                       int64_t w_stride, cudaStream_t stream) {
    auto kern = proj_decode_kernel<EPI, HD>;
    int rc = prepare_kernel<EPI, HD>();
    if (rc) return rc;
    const int n_tiles = (prm.N + kPRows - 1) / kPRows;
    const int split = choose_split<EPI, HD>(n_tiles, prm.kblocks);
    prm.split = split;
    prm.stage_bytes = kPWTile + (uint32_t)prm.Mt * kPK * 2;  // multiple of 2 KiB
    prm.stages = (int)(kPRingBytes / (kPGroupKB * prm.stage_bytes));
    if (prm.stages > kPMaxStages) prm.stages = kPMaxStages;
    prm.w = (const bf16 *)w;
    prm.x = (const bf16 *)x;
    prm.w_stride = w_stride;
    prm.x_stride = x_stride;
    const int mode = dependent_launch_mode();
    prm.pdl_mode = mode;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_tiles * split);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = kPSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = mode > 0 ? 2 : 1;
    if (cudaLaunchKernelEx(&cfg, kern, prm) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    return LC_OK;
}

}  // namespace

int decode_proj_launch(const DecodeProjArgs &a, cudaStream_t stream) {
    if (a.M <= 0 || a.M > kDecodeProjMaxRows || a.K <= 0 || a.N <= 0) return LC_ERR_INVALID_ARGUMENT;
    DecProjParams p{};
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.Mt = (a.M + 15) & ~15;
    p.kblocks = (a.K + kPK - 1) / kPK;
    p.out = (bf16 *)a.out;
    p.out_stride = a.out_stride;
    p.residual = (const bf16 *)a.residual;
    p.res_stride = a.res_stride;
    p.tokens_per_seq = a.tokens_per_seq;
    p.positions = a.positions;
    p.q_bias = (const bf16 *)a.q_bias;
    p.k_bias = (const bf16 *)a.k_bias;
    p.v_bias = (const bf16 *)a.v_bias;
    p.cos_t = a.cos_t;
    p.sin_t = a.sin_t;
    p.rope_rows = a.rope_rows;
    p.k_pool = (bf16 *)a.k_pool;
    p.v_pool = (bf16 *)a.v_pool;
    p.num_blocks = a.num_blocks;
    p.num_layers = a.num_layers;
    p.layer = a.layer;
    p.num_q_heads = a.num_q_heads;
    p.num_kv_heads = a.num_kv_heads;
    p.head_dim = a.head_dim;
    p.tables = a.tables;
    p.table_stride = a.table_stride;
    p.status = a.status;
    if (a.epi == kDecQkv)
        return a.head_dim == 64
                   ? launch_decode_proj<kDecQkv, 64>(p, a.x, a.x_stride, a.w, a.w_stride, stream)
                   : launch_decode_proj<kDecQkv, 128>(p, a.x, a.x_stride, a.w, a.w_stride, stream);
    if (a.epi == kDecResidual)
        return launch_decode_proj<kDecResidual, 128>(p, a.x, a.x_stride, a.w, a.w_stride, stream);
    return launch_decode_proj<kDecPlain, 128>(p, a.x, a.x_stride, a.w, a.w_stride, stream);
}

}  // namespace lc

using namespace lc;

extern "C" int lc_proj_decode_plan(int N, int K, int *split, int *ctas, int *clusters_that_fit,
                                   int *ctas_per_sm_out) {
    if (N <= 0 || K <= 0 || !split || !ctas) return LC_ERR_INVALID_ARGUMENT;
    int rc = prepare_kernel<kDecPlain, 128>();
    if (rc) return rc;
    if (ctas_per_sm_out) *ctas_per_sm_out = ctas_per_sm<kDecPlain, 128>();
    const int n_tiles = (N + kPRows - 1) / kPRows;
    *split = choose_split<kDecPlain, 128>(n_tiles, (K + kPK - 1) / kPK);
    *ctas = n_tiles * *split;
    if (clusters_that_fit) *clusters_that_fit = max_clusters<kDecPlain, 128>(*split);
    return LC_OK;
}
