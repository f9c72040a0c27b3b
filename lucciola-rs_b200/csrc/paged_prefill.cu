// paged_prefill.cu - causal prefill attention over the paged KV pool on the
// 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// The reference prefills token by token: rope -> append -> flash-decoding once
// per prompt token (src/models.rs:486-550), i.e. T serial decode launches per
// layer. Here the prompt's K/V are appended first (lc_rope_append with T rows)
// and one launch computes causal attention for every query:
//   out[b, i, h] = softmax_{t <= start_b + i}(q_i . k_t * scale) . v_t
// over cache positions 0..start_b + i (prior context plus the prompt so far).
//
// One CTA per (256-query block, query head, sequence), heaviest blocks first.
// The block is two 128-query tiles that share every K/V tile:
//   warp 0     TMA: both Q tiles once; K and V tiles of 128 keys = 8 pages
//              each, page by page through the block table, into a 2-4 stage
//              ring (128-byte swizzle, completion on mbarriers).
//   warp 1     MMA issuer (one thread), bf16 x bf16 -> fp32 tcgen05.mma, M = 128:
//              S_t = Q_t K_j^T into TMEM (128 columns per tile t), and
//              O_t += P_t V_j with P_t read from TMEM, where softmax wrote it
//              as bf16 over the first 64 columns of S_t. Per K/V tile the
//              order is PV_0, S_0 (next tile), PV_1, S_1 (next tile), so while
//              one softmax warpgroup works the tensor core runs the other
//              tile's products (ping-pong).
//   warps 2-5  softmax warpgroup of Q tile 0, warps 6-9 of Q tile 1: one
//              thread per query row (its TMEM lane): scale, causal mask,
//              running max with lazy rescaling (O is rescaled in TMEM only when
//              a row max grows by more than 2^8), P = 2^(s - m) into TMEM,
//              and at the end O / l -> bf16 output.
// TMEM (512 columns): S/P of tile t at [128 t, 128 t + 128), O of tile t at
// [256 + hd t, 256 + hd (t + 1)).
// GQA: the CTAs of the q heads of one kv head read the same K/V tiles; they
// fit in L2 (a 4 x 4096-token 1.5B prompt holds 16 MB of K/V per layer).
#include "lc_common.cuh"
#include "lc_host.h"
#include "lc_tcgen05.cuh"

namespace lc {
namespace {

constexpr int kBM = 128;  // queries per Q tile (one TMEM lane each)
constexpr int kQT = 2;    // Q tiles per CTA
constexpr int kBN = 128;  // keys per K/V tile (8 pages)
constexpr int kThreadsPf = (3 + 4 * kQT) * 32;  // K/Q TMA, MMA, softmax x 8, V TMA
constexpr int kVWarp = 2 + 4 * kQT;               // warp 10: V TMA
constexpr uint32_t kTmemCols = 512;
// A row is rescaled only when its scores outgrow the reference max by more than
// 2^kGrowLog2: P then stays below 2^64 in bf16, and O and l (fp32) below 2^100.
constexpr float kGrowSum = 18446744073709551616.f;  // 2^64

template <int HD>
struct PrefillCfg {
    static constexpr int kHalves = HD / 64;
    static constexpr int kQBytes = kBM * HD * 2;     // one Q tile
    static constexpr int kTileBytes = kBN * HD * 2;  // one K or V tile
    // K is released as soon as both S products of a tile are done, V only
    // after both PV products: K gets the deeper ring.
    static constexpr int kKStages = HD == 64 ? 4 : 3;
    static constexpr int kVStages = HD == 64 ? 4 : 2;
    static constexpr int kKOff = kQT * kQBytes;
    static constexpr int kVOff = kKOff + kKStages * kTileBytes;
    static constexpr int kSmem = kVOff + kVStages * kTileBytes + 1024;
    static constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, 0);   // B = K tile, K-major
    static constexpr uint32_t kIdescPV = idesc_bf16_f32(kBM, HD, 1);   // B = V tile, MN-major
    static constexpr uint32_t kOCol = kQT * kBN;                       // first O column
    static_assert(kOCol + kQT * HD <= kTmemCols, "TMEM budget");
};

struct PrefillParams {
    bf16 *out;
    int64_t out_stride;
    const int *tables;
    int table_stride;
    const int *start_pos;
    int batch, tokens;
    int64_t pool_rows, num_blocks;
    int num_layers, layer, num_q_heads, num_kv_heads, group, n_qblocks;
    float scale_log2;
    int *status;
};

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float fast_exp2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Softmax helpers, one thread per query row over the 128 columns of its S
// row in TMEM (32 at a time). Keys with index > kq are masked when DIAG.
// row_max: the raw (unscaled) row max.
template <bool DIAG>
__device__ __forceinline__ float row_max(uint32_t tS, int kq) {
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + 32 * c, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float v = (DIAG && 32 * c + i > kq) ? -INFINITY : u2f(r[i]);
            mx[i & 3] = fmaxf(mx[i & 3], v);
        }
    }
    return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

// row_exp: P = 2^(s * scale - m) with one FFMA and one ex2 per score (masked
// scores are -inf and give 0), packed as bf16 pairs into w (keys 2c, 2c + 1 in
// w[c]). Returns their fp32 sum.
template <bool DIAG>
__device__ __forceinline__ void exp_chunk(const uint32_t (&r)[32], int c, int kq, float scale,
                                          float neg_m, uint32_t (&w)[kBN / 2], float (&rs)[4]) {
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        const float s0 = (DIAG && 32 * c + i > kq) ? -INFINITY : u2f(r[i]);
        const float s1 = (DIAG && 32 * c + i + 1 > kq) ? -INFINITY : u2f(r[i + 1]);
        const float e0 = fast_exp2f(fmaf(s0, scale, neg_m));
        const float e1 = fast_exp2f(fmaf(s1, scale, neg_m));
        rs[(i >> 1) & 3] += e0 + e1;
        w[16 * c + (i >> 1)] = pack_bf16(e0, e1);
    }
}

template <bool DIAG>
__device__ __forceinline__ float row_exp(uint32_t tS, int kq, float scale, float neg_m,
                                         uint32_t (&w)[kBN / 2]) {
    static_assert(kBN == 128, "four 32-column chunks");
    float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + 32 * c, r);
        tmem_wait_ld_regs(r);
        exp_chunk<DIAG>(r, c, kq, scale, neg_m, w, rs);
    }
    return (rs[0] + rs[1]) + (rs[2] + rs[3]);
}

template <int HD>
__global__ void __launch_bounds__(kThreadsPf, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
    using Cfg = PrefillCfg<HD>;
    constexpr int SK = Cfg::kKStages, SV = Cfg::kVStages;
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t k_full[SK], k_empty[SK], v_full[SV], v_empty[SV];
    __shared__ __align__(8) uint64_t s_full[kQT], p_full[kQT], pv_done[kQT];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int s_abort;
    extern __shared__ uint8_t smem_raw[];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // heaviest query blocks (most key tiles) first
    const int per_blk = p.num_q_heads * p.batch;
    const int m = p.n_qblocks - 1 - (int)blockIdx.x / per_blk;
    const int rem = (int)blockIdx.x % per_blk;
    const int h = rem % p.num_q_heads, b = rem / p.num_q_heads;
    const int kvh = h / p.group;
    int start = __ldg(p.start_pos + b);
    if (start < 0 || (long long)start + p.tokens > (long long)p.table_stride * kBlockSize) {
        if (tid == 0 && m == 0 && h == 0) set_status(p.status, LC_DEV_BAD_POS);
        start = max(0, min(start, p.table_stride * kBlockSize - p.tokens));
    }
    const int q0 = m * kQT * kBM;
    // per Q tile: query rows, keys [0, kv_end) needed, K/V tiles
    int rows[kQT], nkv[kQT];
    int nkv_all = 0, kv_end_all = 0;
#pragma unroll
    for (int t = 0; t < kQT; ++t) {
        rows[t] = max(0, min(kBM, p.tokens - (q0 + t * kBM)));
        const int kv_end = rows[t] > 0 ? start + q0 + t * kBM + rows[t] : 0;
        nkv[t] = (kv_end + kBN - 1) / kBN;
        if (rows[t] > 0) {
            nkv_all = nkv[t];
            kv_end_all = kv_end;
        }
    }

    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *gen = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t sQ = base, sK = base + Cfg::kKOff, sV = base + Cfg::kVOff;

    if (tid == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < SK; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < SV; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int t = 0; t < kQT; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], kBM / 32);
            mbar_init(&pv_done[t], 1);
        }
        s_abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_sh, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp == 0 || warp == kVWarp) {
        // ------------------------------------------------------------ TMA --
        // Warp 0 loads both Q tiles and the K tiles, warp 10 the V tiles; each
        // K or V tile is 8 pages found through the block table.
        if (lane == 0) {
            const bool is_k = warp == 0;
            const CUtensorMap *tm = is_k ? &tm_k : &tm_v;
            prefetch_tensormap(tm);
            if (is_k) {
                prefetch_tensormap(&tm_q);
                int nq = 0;
#pragma unroll
                for (int t = 0; t < kQT; ++t) nq += rows[t] > 0;
                mbar_arrive_expect_tx(&q_full, (uint32_t)(nq * Cfg::kQBytes));
#pragma unroll
                for (int t = 0; t < kQT; ++t)
                    if (rows[t] > 0)
#pragma unroll
                        for (int hh = 0; hh < Cfg::kHalves; ++hh)
                            tma_load_2d(gen + t * Cfg::kQBytes + hh * 16384, &tm_q, h * HD + hh * 64,
                                        b * p.tokens + q0 + t * kBM, &q_full);
            }
            const int ns = is_k ? SK : SV;
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            const int off = is_k ? Cfg::kKOff : Cfg::kVOff;
            const int *trow = p.tables + (int64_t)b * p.table_stride;
            const int pages_needed = (kv_end_all + kBlockSize - 1) / kBlockSize;
            for (int j = 0; j < nkv_all; ++j) {
                const int s = j % ns;
                if (j >= ns &&
                    !mbar_wait_bounded(&empty[s], ((j / ns) - 1) & 1, &s_abort, p.status))
                    break;
                int64_t prow[kBN / kBlockSize];
#pragma unroll
                for (int pg = 0; pg < kBN / kBlockSize; ++pg) {
                    const int logical = j * (kBN / kBlockSize) + pg;
                    const int phys = logical < pages_needed ? __ldg(trow + logical) : -1;
                    if (phys >= 0 && phys < p.num_blocks) {
                        prow[pg] = page_row(phys, p.layer, kvh, p.num_layers, p.num_kv_heads);
                    } else {
                        if (is_k && logical < pages_needed) set_status(p.status, LC_DEV_BAD_BLOCK);
                        prow[pg] = p.pool_rows;  // wholly out of bounds: zero fill
                    }
                }
                mbar_arrive_expect_tx(&full[s], Cfg::kTileBytes);
#pragma unroll
                for (int pg = 0; pg < kBN / kBlockSize; ++pg)
#pragma unroll
                    for (int hh = 0; hh < Cfg::kHalves; ++hh)
                        tma_load_2d(gen + off + s * Cfg::kTileBytes + hh * 16384 + pg * 2048, tm,
                                    hh * 64, (int)prow[pg], &full[s]);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA --
        if (lane == 0) {
            bool ok = mbar_wait_bounded(&q_full, 0, &s_abort, p.status);
            int k_ready = -1;  // K tiles up to this one have landed
            auto wait_k = [&](int j) -> bool {
                if (j <= k_ready) return true;
                if (!mbar_wait_bounded(&k_full[j % SK], (j / SK) & 1, &s_abort, p.status)) return false;
                k_ready = j;
                return true;
            };
            auto issue_s = [&](int t, int j) {
                tc_fence_after();
                const uint32_t kt = sK + (j % SK) * Cfg::kTileBytes, qt = sQ + t * Cfg::kQBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16(tmem + t * kBN, sw128_desc(qt + off, 16, 1024),
                              sw128_desc(kt + off, 16, 1024), Cfg::kIdescS, kk > 0);
                }
                umma_commit(&s_full[t]);
            };
            auto issue_pv = [&](int t, int j) {
                tc_fence_after();
                const uint32_t vt = sV + (j % SV) * Cfg::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                    umma_bf16_tmem_a(tmem + Cfg::kOCol + t * HD, tmem + t * kBN + kk * 8,
                                     sw128_desc(vt + kk * 2048, 16384, 1024), Cfg::kIdescPV,
                                     (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&pv_done[t]);
            };
            if (ok && nkv_all > 0) ok = wait_k(0);
#pragma unroll
            for (int t = 0; t < kQT; ++t)
                if (ok && nkv[t] > 0) issue_s(t, 0);
            if (ok && nkv_all > 0) umma_commit(&k_empty[0]);  // K(0) is done once both S(0) are
            for (int j = 0; j < nkv_all && ok; ++j) {
                bool v_ready = false;
#pragma unroll
                for (int t = 0; t < kQT; ++t) {
                    if (!ok || j >= nkv[t]) continue;
                    if (!mbar_wait_bounded(&p_full[t], j & 1, &s_abort, p.status)) {
                        ok = false;
                        break;
                    }
                    if (!v_ready) {
                        if (!mbar_wait_bounded(&v_full[j % SV], (j / SV) & 1, &s_abort, p.status)) {
                            ok = false;
                            break;
                        }
                        v_ready = true;
                    }
                    // PV_t reads P_t from the columns S_t(j + 1) then overwrites;
                    // MMAs of one thread run in issue order.
                    issue_pv(t, j);
                    if (j + 1 < nkv[t]) {
                        if (!wait_k(j + 1)) {
                            ok = false;
                            break;
                        }
                        issue_s(t, j + 1);
                    }
                }
                if (!ok) break;
                umma_commit(&v_empty[j % SV]);                            // both PV(j) issued
                if (j + 1 < nkv_all) umma_commit(&k_empty[(j + 1) % SK]);  // both S(j + 1) issued
            }
        }
    } else {
        // -------------------------------------------------------- softmax --
        const int t = (warp - 2) >> 2;  // Q tile of this warpgroup (warps 2-9)
        static_assert(kQT == 2, "per-tile values below are selected for two tiles");
        const int my_rows = t ? rows[1] : rows[0];
        const int my_nkv = t ? nkv[1] : nkv[0];
        const int quad = warp & 3;       // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t tS = tl + t * kBN, tO = tl + Cfg::kOCol + t * HD;
        const int q_idx = q0 + t * kBM + row;
        const int q_pos = start + q_idx;
        const int first_q = start + q0 + t * kBM;  // position of the tile's first query
        float m_ref = -INFINITY, l = 0.f;
        bool ok = my_rows > 0;
        for (int j = 0; j < my_nkv && ok; ++j) {
            if (!mbar_wait_bounded(&s_full[t], j & 1, &s_abort, p.status)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int key0 = j * kBN;
            // Causal mask only on tiles that reach past the tile's first query.
            const bool diag = key0 + kBN - 1 > first_q;
            const int kq = q_pos - key0;  // keys of the tile past this index are masked
            // The first tile sets the reference max m_ref (a max pass first).
            // Later tiles exponentiate against it in one pass with no max at
            // all: a row whose scores outgrew m_ref by more than 2^kGrowLog2
            // shows it in its sum (inf included); then its true max is taken,
            // O and l are rescaled and the row is redone (S is intact in TMEM).
            uint32_t w[kBN / 2];
            float alpha = 1.f, sum = 0.f;
            bool rescale = false, grew = false, need_max = j == 0;
#pragma unroll 1
            for (int pass = 0; pass < 2; ++pass) {
                if (need_max) {
                    const float mt =
                        (diag ? row_max<true>(tS, kq) : row_max<false>(tS, kq)) * p.scale_log2;
                    if (j == 0) {
                        m_ref = mt;
                    } else if (grew) {
                        alpha = fast_exp2f(m_ref - mt);
                        m_ref = mt;
                        rescale = true;
                    }
                }
                sum = diag ? row_exp<true>(tS, kq, p.scale_log2, -m_ref, w)
                           : row_exp<false>(tS, kq, p.scale_log2, -m_ref, w);
                grew = !(sum <= kGrowSum);
                if (!__any_sync(0xffffffffu, grew)) break;
                need_max = true;
            }
            l = l * alpha + sum;

            if (__any_sync(0xffffffffu, rescale)) {
                // O may be rescaled once PV(j - 1) is done with it.
                if (!mbar_wait_bounded(&pv_done[t], (j - 1) & 1, &s_abort, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tO + 32 * c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = f2u(u2f(r[i]) * alpha);
                    tmem_st32(tO + 32 * c, r);
                }
            }
            // Keys past the prompt end in the CTA's last K/V tile: zero their V
            // rows so that 0 * (stale or non-finite pool contents) cannot reach
            // O. Each warpgroup that uses the tile does so before its PV.
            if (j == nkv_all - 1 && kv_end_all < key0 + kBN) {
                const int s = j % SV;
                if (!mbar_wait_bounded(&v_full[s], (j / SV) & 1, &s_abort, p.status)) {
                    ok = false;
                    break;
                }
                if (row >= kv_end_all - key0) {
#pragma unroll
                    for (int hh = 0; hh < Cfg::kHalves; ++hh)
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<uint4 *>(gen + Cfg::kVOff + s * Cfg::kTileBytes +
                                                       hh * 16384 + row * 128 + c * 16) =
                                make_uint4(0, 0, 0, 0);
                }
                fence_proxy_async_smem();
            }
            // P as bf16 pairs over the first 64 columns of S (keys 2c, 2c + 1 in
            // column c): the A operand of PV.
            tmem_st32(tS, *reinterpret_cast<const uint32_t(*)[32]>(&w[0]));
            tmem_st32(tS + 32, *reinterpret_cast<const uint32_t(*)[32]>(&w[32]));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);  // one arrival per warp
        }
        // ----------------------------------------------------- epilogue --
        if (ok && mbar_wait_bounded(&pv_done[t], (my_nkv - 1) & 1, &s_abort, p.status)) {
            tc_fence_after();
            const float inv = 1.f / l;
            bf16 *orow = p.out + (int64_t)(b * p.tokens + q_idx) * p.out_stride + (int64_t)h * HD;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tO + 32 * c, r);
                tmem_wait_ld();
                if (q_idx < p.tokens) {
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint4 o;
                        o.x = pack_bf16(u2f(r[8 * v + 0]) * inv, u2f(r[8 * v + 1]) * inv);
                        o.y = pack_bf16(u2f(r[8 * v + 2]) * inv, u2f(r[8 * v + 3]) * inv);
                        o.z = pack_bf16(u2f(r[8 * v + 4]) * inv, u2f(r[8 * v + 5]) * inv);
                        o.w = pack_bf16(u2f(r[8 * v + 6]) * inv, u2f(r[8 * v + 7]) * inv);
                        *reinterpret_cast<uint4 *>(orow + 32 * c + 8 * v) = o;
                    }
                }
            }
        }
    }
    // ------------------------------------------------------------ teardown --
    if (s_abort && warp == 0 && lane == 0) {
        // a wait gave up: let the copies in flight land before the CTA exits
        mbar_wait_drain(&q_full, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <int HD>
int launch_prefill(const PrefillParams &prm, const void *q, int64_t q_stride,
                   const void *k_pool, const void *v_pool, cudaStream_t stream) {
    CUtensorMap mq, mk, mv;
    int rc = tensor_map_2d_sw128(q, (int64_t)prm.num_q_heads * HD,
                                 (int64_t)prm.batch * prm.tokens, q_stride * 2, 64, kBM, &mq);
    if (rc) return rc;
    rc = pool_tensor_map(k_pool, prm.pool_rows, HD, &mk);
    if (rc) return rc;
    rc = pool_tensor_map(v_pool, prm.pool_rows, HD, &mv);
    if (rc) return rc;
    const int smem = PrefillCfg<HD>::kSmem;
    rc = ensure_smem_attr((const void *)paged_prefill_kernel<HD>, smem);
    if (rc) return rc;
    const unsigned grid = (unsigned)prm.n_qblocks * prm.num_q_heads * prm.batch;
    paged_prefill_kernel<HD><<<grid, kThreadsPf, smem, stream>>>(mq, mk, mv, prm);
    return launch_status();
}

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" int lc_paged_prefill(void *out, int64_t out_stride, const void *q, int64_t q_stride,
                                const void *k_pool, const void *v_pool, int64_t num_blocks,
                                int num_layers, int layer, int num_q_heads, int num_kv_heads,
                                int head_dim, const int *block_tables, int table_stride,
                                const int *start_pos, int num_seqs, int tokens_per_seq,
                                int max_start_pos, float sm_scale, int *dev_status,
                                lc_stream_t stream) {
    (void)max_start_pos;  // positions are read on the device
    if (!out || !q || !k_pool || !v_pool || !block_tables || !start_pos)
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (num_seqs < 0 || tokens_per_seq < 0 || num_layers <= 0 || layer < 0 ||
        layer >= num_layers || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
        table_stride <= 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if (num_seqs == 0 || tokens_per_seq == 0) return LC_OK;
    if ((int64_t)num_seqs * tokens_per_seq >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;
    if (!aligned16(k_pool) || !aligned16(v_pool) || !aligned16(q) || !aligned16(out) ||
        (q_stride & 7) || (out_stride & 7))
        return LC_ERR_MISALIGNED;
    if (q_stride < (int64_t)num_q_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim)
        return LC_ERR_INVALID_ARGUMENT;
    const int64_t pool_rows = num_blocks * num_layers * num_kv_heads * kBlockSize;
    if (pool_rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;
    const int64_t n_qblocks = (tokens_per_seq + kQT * kBM - 1) / (kQT * kBM);
    if (n_qblocks * num_q_heads * num_seqs >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;

    PrefillParams prm{};
    prm.out = (bf16 *)out;
    prm.out_stride = out_stride;
    prm.tables = block_tables;
    prm.table_stride = table_stride;
    prm.start_pos = start_pos;
    prm.batch = num_seqs;
    prm.tokens = tokens_per_seq;
    prm.pool_rows = pool_rows;
    prm.num_blocks = num_blocks;
    prm.num_layers = num_layers;
    prm.layer = layer;
    prm.num_q_heads = num_q_heads;
    prm.num_kv_heads = num_kv_heads;
    prm.group = num_q_heads / num_kv_heads;
    prm.n_qblocks = (int)n_qblocks;
    prm.scale_log2 = sm_scale * 1.4426950408889634f;
    prm.status = dev_status;
    cudaStream_t s = as_stream(stream);
    return head_dim == 64 ? launch_prefill<64>(prm, q, q_stride, k_pool, v_pool, s)
                          : launch_prefill<128>(prm, q, q_stride, k_pool, v_pool, s);
}
