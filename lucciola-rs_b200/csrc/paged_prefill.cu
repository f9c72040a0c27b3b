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
// One CTA per (128-query tile, query head, sequence), heaviest tiles first.
//   warp 0    TMA: the Q tile once; K and V tiles of 128 keys = 8 pages each,
//             page by page through the block table, into a 2-3 stage ring
//             (128-byte swizzle, completion on mbarriers).
//   warp 1    MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM S
//             buffers (128 x 128 fp32), then O += P_j V_j into TMEM O
//             (128 x hd fp32); both bf16 x bf16 -> fp32 tcgen05.mma, M = 128.
//             S_{j+1} is issued before PV_j so softmax j+1 overlaps PV_j.
//   warps 2-5 softmax, one thread per query row (its TMEM lane): scale, causal
//             mask, running max with lazy rescaling (O is rescaled in TMEM only
//             when a row max grows by more than 2^8), P_j = 2^(s - m) as bf16
//             into shared memory for the PV MMA, then O / l -> bf16 output.
// GQA: the CTAs of the q heads of one kv head read the same K/V tiles; they
// fit in L2 (a 4 x 4096-token 1.5B prompt holds 16 MB of K/V per layer).
#include "lc_common.cuh"
#include "lc_host.h"
#include "lc_tcgen05.cuh"

namespace lc {
namespace {

constexpr int kBM = 128;  // queries per CTA
constexpr int kBN = 128;  // keys per tile (8 pages)
constexpr int kThreadsPf = 192;
constexpr uint32_t kTmemCols = 512;       // S0 [0,128) S1 [128,256) O [256, 256+hd)
constexpr float kRescaleLog2 = 8.f;       // rescale O only when a row max grows by > 2^8

template <int HD>
struct PrefillCfg {
    static constexpr int kHalves = HD / 64;
    static constexpr int kQBytes = kBM * HD * 2;
    static constexpr int kTileBytes = kBN * HD * 2;  // one K or V tile
    static constexpr int kStages = HD == 64 ? 3 : 2;
    static constexpr int kPBytes = kBM * kBN * 2;
    static constexpr int kKOff = kQBytes;
    static constexpr int kVOff = kKOff + kStages * kTileBytes;
    static constexpr int kPOff = kVOff + kStages * kTileBytes;  // two P buffers
    static constexpr int kSmem = kPOff + 2 * kPBytes + 1024;
    static constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, 0);   // B = K tile, K-major
    static constexpr uint32_t kIdescPV = idesc_bf16_f32(kBM, HD, 1);   // B = V tile, MN-major
};

struct PrefillParams {
    bf16 *out;
    int64_t out_stride;
    const int *tables;
    int table_stride;
    const int *start_pos;
    int batch, tokens;
    int64_t pool_rows, num_blocks;
    int num_layers, layer, num_q_heads, num_kv_heads, group, n_qtiles;
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

template <int HD>
__global__ void __launch_bounds__(kThreadsPf, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
    using Cfg = PrefillCfg<HD>;
    constexpr int S = Cfg::kStages;
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t k_full[S], v_full[S], kv_empty[S];
    __shared__ __align__(8) uint64_t s_full[2], s_free[2];
    __shared__ __align__(8) uint64_t p_full[2], pv_done[2];  // per P buffer: tile t uses t % 2
    __shared__ uint32_t tmem_base_sh;
    __shared__ int s_abort;
    extern __shared__ uint8_t smem_raw[];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // heaviest query tiles (most key tiles) first
    const int per_tile = p.num_q_heads * p.batch;
    const int m = p.n_qtiles - 1 - (int)blockIdx.x / per_tile;
    const int rem = (int)blockIdx.x % per_tile;
    const int h = rem % p.num_q_heads, b = rem / p.num_q_heads;
    const int kvh = h / p.group;
    int start = __ldg(p.start_pos + b);
    const int q0 = m * kBM;
    const int q_rows = min(kBM, p.tokens - q0);
    if (start < 0 || (long long)start + p.tokens > (long long)p.table_stride * kBlockSize) {
        if (tid == 0 && m == 0 && h == 0) set_status(p.status, LC_DEV_BAD_POS);
        start = max(0, min(start, p.table_stride * kBlockSize - p.tokens));
    }
    const int kv_end = start + q0 + q_rows;  // keys [0, kv_end) are needed
    const int nkv = (kv_end + kBN - 1) / kBN;

    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *gen = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t sQ = base, sK = base + Cfg::kKOff, sV = base + Cfg::kVOff, sP = base + Cfg::kPOff;

    if (tid == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < S; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], kBM);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&p_full[i], kBM);
            mbar_init(&pv_done[i], 1);
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

    if (warp == 0) {
        // ------------------------------------------------------------ TMA --
        if (lane == 0) {
            prefetch_tensormap(&tm_q);
            prefetch_tensormap(&tm_k);
            prefetch_tensormap(&tm_v);
            mbar_arrive_expect_tx(&q_full, Cfg::kQBytes);
#pragma unroll
            for (int hh = 0; hh < Cfg::kHalves; ++hh)
                tma_load_2d(gen + hh * 16384, &tm_q, h * HD + hh * 64, b * p.tokens + q0, &q_full);
            const int *trow = p.tables + (int64_t)b * p.table_stride;
            const int pages_needed = (kv_end + kBlockSize - 1) / kBlockSize;
            for (int j = 0; j < nkv; ++j) {
                const int s = j % S;
                if (j >= S &&
                    !mbar_wait_bounded(&kv_empty[s], ((j / S) - 1) & 1, &s_abort, p.status))
                    break;
                int64_t rows[kBN / kBlockSize];
#pragma unroll
                for (int pg = 0; pg < kBN / kBlockSize; ++pg) {
                    const int logical = j * (kBN / kBlockSize) + pg;
                    const int phys = logical < pages_needed ? __ldg(trow + logical) : -1;
                    if (phys >= 0 && phys < p.num_blocks) {
                        rows[pg] = page_row(phys, p.layer, kvh, p.num_layers, p.num_kv_heads);
                    } else {
                        if (logical < pages_needed) set_status(p.status, LC_DEV_BAD_BLOCK);
                        rows[pg] = p.pool_rows;  // wholly out of bounds: zero fill
                    }
                }
                mbar_arrive_expect_tx(&k_full[s], Cfg::kTileBytes);
#pragma unroll
                for (int pg = 0; pg < kBN / kBlockSize; ++pg)
#pragma unroll
                    for (int hh = 0; hh < Cfg::kHalves; ++hh)
                        tma_load_2d(gen + Cfg::kKOff + s * Cfg::kTileBytes + hh * 16384 + pg * 2048,
                                    &tm_k, hh * 64, (int)rows[pg], &k_full[s]);
                mbar_arrive_expect_tx(&v_full[s], Cfg::kTileBytes);
#pragma unroll
                for (int pg = 0; pg < kBN / kBlockSize; ++pg)
#pragma unroll
                    for (int hh = 0; hh < Cfg::kHalves; ++hh)
                        tma_load_2d(gen + Cfg::kVOff + s * Cfg::kTileBytes + hh * 16384 + pg * 2048,
                                    &tm_v, hh * 64, (int)rows[pg], &v_full[s]);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA --
        if (lane == 0) {
            bool ok = mbar_wait_bounded(&q_full, 0, &s_abort, p.status);
            tc_fence_after();
            auto issue_s = [&](int j) -> bool {
                const int s = j % S;
                if (!mbar_wait_bounded(&k_full[s], (j / S) & 1, &s_abort, p.status)) return false;
                if (j >= 2 &&
                    !mbar_wait_bounded(&s_free[j & 1], ((j >> 1) - 1) & 1, &s_abort, p.status))
                    return false;
                tc_fence_after();
                const uint32_t kt = sK + s * Cfg::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16(tmem + (j & 1) * kBN, sw128_desc(sQ + off, 16, 1024),
                              sw128_desc(kt + off, 16, 1024), Cfg::kIdescS, kk > 0);
                }
                umma_commit(&s_full[j & 1]);
                return true;
            };
            auto issue_pv = [&](int t) -> bool {
                const int s = t % S;
                if (!mbar_wait_bounded(&p_full[t & 1], (t >> 1) & 1, &s_abort, p.status)) return false;
                if (!mbar_wait_bounded(&v_full[s], (t / S) & 1, &s_abort, p.status)) return false;
                tc_fence_after();
                const uint32_t vt = sV + s * Cfg::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                    const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16(tmem + 2 * kBN, sw128_desc(sP + (t & 1) * Cfg::kPBytes + aoff, 16, 1024),
                              sw128_desc(vt + kk * 2048, 16384, 1024), Cfg::kIdescPV,
                              (t > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&pv_done[t & 1]);
                umma_commit(&kv_empty[s]);
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 1; j < nkv && ok; ++j) ok = issue_s(j) && issue_pv(j - 1);
            if (ok) ok = issue_pv(nkv - 1);
            // Let every MMA this thread issued finish before the teardown.
            if (ok) mbar_wait_bounded(&pv_done[(nkv - 1) & 1], ((nkv - 1) >> 1) & 1, &s_abort, p.status);
        }
    } else {
        // -------------------------------------------------------- softmax --
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        const int q_idx = q0 + row;
        const int q_pos = start + q_idx;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv && ok; ++j) {
            if (!mbar_wait_bounded(&s_full[j & 1], (j >> 1) & 1, &s_abort, p.status)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[kBN];
            {
                uint32_t r[kBN / 32][32];
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) tmem_ld32(tl + (j & 1) * kBN + 32 * c, r[c]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i) sv[32 * c + i] = u2f(r[c][i]);
            }
            tc_fence_before();
            mbar_arrive(&s_free[j & 1]);
            const int key0 = j * kBN;
            // Causal mask only on tiles that reach past the tile's first query.
            if (key0 + kBN - 1 > start + q0) {
#pragma unroll
                for (int c = 0; c < kBN; ++c)
                    if (key0 + c > q_pos) sv[c] = -INFINITY;
            }
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < kBN; ++c) mx[c & 3] = fmaxf(mx[c & 3], sv[c]);
            // raw scores: scale > 0 keeps the order, so scale the max only
            const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * p.scale_log2;
            // Running max with lazy rescaling: keep the reference max unless the
            // tile's max exceeds it by more than 2^8; then O and l are rescaled.
            float alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m_ref = mt;
            } else if (mt > m_ref + kRescaleLog2) {
                alpha = fast_exp2f(m_ref - mt);
                m_ref = mt;
                rescale = true;
            }
            // P = 2^(s * scale - m_ref) (masked keys give 0): one FFMA and one
            // ex2 per score, computed before any wait.
            float rs[4] = {0.f, 0.f, 0.f, 0.f};
            const float neg_m = -m_ref;
#pragma unroll
            for (int c = 0; c < kBN; ++c) {
                sv[c] = fast_exp2f(fmaf(sv[c], p.scale_log2, neg_m));
                rs[c & 3] += sv[c];
            }
            l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
            // P buffer j % 2 is free once PV_{j-2} is done; O may be rescaled
            // only after PV_{j-1}.
            if (j >= 2 &&
                !mbar_wait_bounded(&pv_done[j & 1], ((j - 2) >> 1) & 1, &s_abort, p.status)) {
                ok = false;
                break;
            }
            const bool warp_rescale = __any_sync(0xffffffffu, rescale);
            if (warp_rescale) {
                if (!mbar_wait_bounded(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, &s_abort,
                                       p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tl + 2 * kBN + 32 * c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = f2u(u2f(r[i]) * alpha);
                    tmem_st32(tl + 2 * kBN + 32 * c, r);
                }
                tmem_wait_st();
            }
            // P row in bf16, 128-byte swizzled, K-major (keys).
            uint8_t *pb = gen + Cfg::kPOff + (j & 1) * Cfg::kPBytes;
#pragma unroll
            for (int c16 = 0; c16 < kBN / 8; ++c16) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) w[e] = pack_bf16(sv[8 * c16 + 2 * e], sv[8 * c16 + 2 * e + 1]);
                const int hh = c16 >> 3, cc = c16 & 7;
                *reinterpret_cast<uint4 *>(pb + hh * 16384 + row * 128 + ((cc ^ (row & 7)) << 4)) =
                    make_uint4(w[0], w[1], w[2], w[3]);
            }
            // Keys past the prompt end in the last tile: zero their V rows so
            // that 0 * (stale or non-finite pool contents) cannot reach O.
            if (j == nkv - 1 && kv_end < key0 + kBN) {
                const int s = j % S;
                if (!mbar_wait_bounded(&v_full[s], (j / S) & 1, &s_abort, p.status)) {
                    ok = false;
                    break;
                }
                if (row >= kv_end - key0) {
#pragma unroll
                    for (int hh = 0; hh < Cfg::kHalves; ++hh)
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<uint4 *>(gen + Cfg::kVOff + s * Cfg::kTileBytes +
                                                       hh * 16384 + row * 128 + c * 16) =
                                make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&p_full[j & 1]);
        }
        // ----------------------------------------------------- epilogue --
        if (ok && mbar_wait_bounded(&pv_done[(nkv - 1) & 1], ((nkv - 1) >> 1) & 1, &s_abort,
                                    p.status)) {
            tc_fence_after();
            const float inv = 1.f / l;
            bf16 *orow = p.out + (int64_t)(b * p.tokens + q_idx) * p.out_stride + (int64_t)h * HD;
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tl + 2 * kBN + 32 * c, r);
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
    const unsigned grid = (unsigned)prm.n_qtiles * prm.num_q_heads * prm.batch;
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
    const int64_t n_qtiles = (tokens_per_seq + kBM - 1) / kBM;
    if (n_qtiles * num_q_heads * num_seqs >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;

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
    prm.n_qtiles = (int)n_qtiles;
    prm.scale_log2 = sm_scale * 1.4426950408889634f;
    prm.status = dev_status;
    cudaStream_t s = as_stream(stream);
    return head_dim == 64 ? launch_prefill<64>(prm, q, q_stride, k_pool, v_pool, s)
                          : launch_prefill<128>(prm, q, q_stride, k_pool, v_pool, s);
}
