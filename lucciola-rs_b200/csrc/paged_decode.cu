// paged_decode.cu - batched paged flash-decoding attention for GQA (sm_100a).
//
// Replaces flash_decoding_kernel_64/128 (src/kernels/attention.cu:4-240), which
// runs one 1024-thread CTA per query head over one sequence and so reads every
// KV byte Hq/Hkv times with scalar 2-byte loads. Here:
//
//  * One CTA per (partition of <= P tokens, kv head [x8-head slice], sequence).
//    The CTA serves all query heads of the kv head's group (up to 8), so each KV
//    byte leaves HBM once.
//  * A producer warp streams the partition's pages into a ring of shared-memory
//    stages with TMA tile loads (one {64 x 16} box per half page, 128-byte
//    swizzle), completion tracked by mbarriers with a transaction count.
//  * Four consumer warps each take one 16-token page per stage and run both
//    products on the tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate)
//    with tokens on M and the <= 8 query heads on N:
//        S^T[16 tok x 8 heads]  = K_page[16 x hd] . Q^T[hd x 8]
//        O^T[hd x 8 heads]     += V_page^T[hd x 16] . P^T[16 x 8]
//    P^T goes from the accumulator layout to the B-operand layout with
//    movmatrix.trans, without touching shared memory. Online softmax in base 2.
//  * Split-K: partitions write (O/l, log2-sum-exp) to the workspace; the last
//    CTA of a (sequence, kv head) to finish (arrival counter) merges them with a
//    warp-shuffle log-sum-exp reduction and writes the bf16 output.
//
// Semantics follow attention.cu: out = softmax(q.k * scale) . v over cache
// tokens 0..n-1, fp32 accumulation, bf16 output. Block-table entries outside
// the pool are reported in the status word and read as zeros (TMA bounds fill).
#include <climits>

#include "lc_common.cuh"
#include "lc_host.h"

namespace lc {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kHeadsPerCta = 8;
constexpr int kMaxPartitions = 256;
constexpr int kPagesPerStage = 4;  // one page per consumer warp per stage

template <int HD>
struct DecodeCfg {
    static constexpr int kPageBytes = kBlockSize * HD * 2;  // 2 KiB / 4 KiB
    static constexpr int kStages = HD == 64 ? 4 : 3;
    static constexpr int kStageBytes = kPagesPerStage * 2 * kPageBytes;  // K pages, V pages
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024;    // + alignment slack
    static_assert(kStages * kStageBytes >=
                      kConsumerWarps * kHeadsPerCta * (HD + 2) * 4 + kHeadsPerCta * (kMaxPartitions + 1) * 4,
                  "merge scratch must fit in the stage ring");
};

struct DecodeParams {
    bf16 *out;
    int64_t out_stride;
    const bf16 *q;
    int64_t q_stride;
    const int *tables;
    int table_stride;
    const int *ctx_lens;
    int len_offset;
    int64_t pool_rows;  // rows of the [rows][hd] pool view; used as an all-out-of-bounds row
    int64_t num_blocks;
    int num_layers, layer, num_q_heads, num_kv_heads, group, ctas_per_kv;
    int partition_tokens;
    float scale_log2;  // sm_scale * log2(e)
    float *ws_o;
    float *ws_lse;
    int *ws_cnt;
    int *status;
};

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Shared-memory byte address of 16-byte chunk `kc` (of hd/8) of token row `r` in a
// page tile stored as hd/64 boxes of [16 rows][128 B] with 128-byte swizzle.
__device__ __forceinline__ uint32_t tile_addr(uint32_t page, int r, int kc) {
    return page + ((kc >> 3) << 11) + (r << 7) + ((((kc & 7) ^ (r & 7))) << 4);
}

template <int HD>
__global__ void __launch_bounds__(kThreads)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const DecodeParams p) {
    using Cfg = DecodeCfg<HD>;
    constexpr int KSTEPS = HD / 16;

    __shared__ __align__(8) uint64_t full_bar[Cfg::kStages];
    __shared__ __align__(8) uint64_t empty_bar[Cfg::kStages];
    __shared__ int s_abort;
    __shared__ int s_last;
    extern __shared__ uint8_t smem_raw[];

    const int b = blockIdx.z;
    const int kvh = blockIdx.y / p.ctas_per_kv;
    const int hsub = blockIdx.y - kvh * p.ctas_per_kv;
    const int head0 = kvh * p.group + hsub * kHeadsPerCta;
    const int nh = min(kHeadsPerCta, p.group - hsub * kHeadsPerCta);
    const int part = blockIdx.x;
    const int tid = threadIdx.x;

    int n = p.ctx_lens[b] + p.len_offset;
    if (n < 0) n = 0;
    const int table_cap = p.table_stride * kBlockSize;
    if (n > table_cap) {
        if (part == 0 && tid == 0) set_status(p.status, LC_DEV_BAD_POS);
        n = table_cap;
    }
    if (n == 0) {  // empty context: defined as a zero output
        if (part == 0)
            for (int i = tid; i < nh * HD; i += kThreads)
                p.out[(int64_t)b * p.out_stride + (int64_t)head0 * HD + i] = __float2bfloat16(0.f);
        return;
    }
    int ptok = p.partition_tokens;
    {
        const int need = ((n + (int)gridDim.x - 1) / (int)gridDim.x + kBlockSize - 1) & ~(kBlockSize - 1);
        if (need > ptok) ptok = need;
    }
    const int nparts = (n + ptok - 1) / ptok;
    if (part >= nparts) return;
    const int t0 = part * ptok;
    const int t1 = min(t0 + ptok, n);
    const int npages = (t1 - t0 + kBlockSize - 1) / kBlockSize;

    const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem_gen = smem_raw + (smem_base - smem_u32(smem_raw));

    if (tid == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kConsumerWarps);
        }
        s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    const int warp = tid >> 5, lane = tid & 31;

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer --
        if (lane == 0) {
            prefetch_tensormap(&tmap_k);
            prefetch_tensormap(&tmap_v);
            const int *trow = p.tables + (int64_t)b * p.table_stride;
            const int first_page = t0 / kBlockSize;
            for (int pg = 0, it = 0; pg < npages; pg += kPagesPerStage, ++it) {
                const int s = it % Cfg::kStages;
                if (it >= Cfg::kStages &&
                    !mbar_wait_bounded(&empty_bar[s], ((it / Cfg::kStages) - 1) & 1, &s_abort,
                                       p.status))
                    break;
                const int np = min(kPagesPerStage, npages - pg);
                mbar_arrive_expect_tx(&full_bar[s], (uint32_t)(np * 2 * Cfg::kPageBytes));
                const uint32_t stage = smem_base + s * Cfg::kStageBytes;
                for (int j = 0; j < np; ++j) {
                    const int phys = __ldg(trow + first_page + pg + j);
                    int64_t row;
                    if (phys < 0 || phys >= p.num_blocks) {
                        set_status(p.status, LC_DEV_BAD_BLOCK);
                        row = p.pool_rows;  // entirely out of bounds: TMA fills zeros
                    } else {
                        row = page_row(phys, p.layer, kvh, p.num_layers, p.num_kv_heads);
                    }
                    uint8_t *kdst = smem_gen + (stage - smem_base) + j * Cfg::kPageBytes;
                    uint8_t *vdst = kdst + kPagesPerStage * Cfg::kPageBytes;
#pragma unroll
                    for (int h = 0; h < HD / 64; ++h) {
                        tma_load_2d(kdst + h * 2048, &tmap_k, h * 64, (int)row, &full_bar[s]);
                        tma_load_2d(vdst + h * 2048, &tmap_v, h * 64, (int)row, &full_bar[s]);
                    }
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------- consumers --
    const int g = lane >> 2, c = lane & 3;
    uint32_t qf[KSTEPS][2];
    {
        const bool hv = g < nh;
        const bf16 *qrow = p.q + (int64_t)b * p.q_stride + (int64_t)(head0 + (hv ? g : 0)) * HD;
#pragma unroll
        for (int j = 0; j < KSTEPS; ++j) {
            qf[j][0] = hv ? __ldg(reinterpret_cast<const uint32_t *>(qrow + 16 * j + 2 * c)) : 0u;
            qf[j][1] = hv ? __ldg(reinterpret_cast<const uint32_t *>(qrow + 16 * j + 8 + 2 * c)) : 0u;
        }
    }
    float o[KSTEPS][4];
#pragma unroll
    for (int i = 0; i < KSTEPS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    // Per-lane ldmatrix row/chunk selectors.
    const int mi = lane >> 3, r8 = lane & 7;
    const int k_row = (mi & 1) * 8 + r8, k_chunk = mi >> 1;  // QK A operand (K tile)
    const int v_row = (mi >> 1) * 8 + r8, v_chunk = mi & 1;  // PV A operand (V^T tile)

    for (int pg = 0, it = 0; pg < npages; pg += kPagesPerStage, ++it) {
        const int s = it % Cfg::kStages;
        if (!mbar_wait_bounded(&full_bar[s], (it / Cfg::kStages) & 1, &s_abort, p.status)) break;
        const int pi = pg + warp;
        if (pi < npages) {
            const int valid = min(kBlockSize, t1 - (t0 + pi * kBlockSize));
            const uint32_t kpage = smem_base + s * Cfg::kStageBytes + warp * Cfg::kPageBytes;
            const uint32_t vpage = kpage + kPagesPerStage * Cfg::kPageBytes;
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < KSTEPS; ++j) {
                uint32_t a[4];
                ldmatrix_x4(a, tile_addr(kpage, k_row, 2 * j + k_chunk));
                mma_bf16_16816(sc, a, qf[j][0], qf[j][1]);
            }
            // sc: (tok g, head 2c), (g, 2c+1), (g+8, 2c), (g+8, 2c+1)
            float s0 = g < valid ? sc[0] * p.scale_log2 : -INFINITY;
            float s1 = g < valid ? sc[1] * p.scale_log2 : -INFINITY;
            float s2 = g + 8 < valid ? sc[2] * p.scale_log2 : -INFINITY;
            float s3 = g + 8 < valid ? sc[3] * p.scale_log2 : -INFINITY;
            float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
            const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
            const float al0 = fast_exp2(m0 - mu0), al1 = fast_exp2(m1 - mu1);
            m0 = mn0;
            m1 = mn1;
            const float p0 = fast_exp2(s0 - mu0), p1 = fast_exp2(s1 - mu1);
            const float p2 = fast_exp2(s2 - mu0), p3 = fast_exp2(s3 - mu1);
            l0 = l0 * al0 + (p0 + p2);
            l1 = l1 * al1 + (p1 + p3);
#pragma unroll
            for (int i = 0; i < KSTEPS; ++i) {
                o[i][0] *= al0;
                o[i][1] *= al1;
                o[i][2] *= al0;
                o[i][3] *= al1;
            }
            const uint32_t b0 = movmatrix_trans(pack_bf16(p0, p1));
            const uint32_t b1 = movmatrix_trans(pack_bf16(p2, p3));
#pragma unroll
            for (int i = 0; i < KSTEPS; ++i) {
                uint32_t a[4];
                ldmatrix_x4_trans(a, tile_addr(vpage, v_row, 2 * i + v_chunk));
                mma_bf16_16816(o[i], a, b0, b1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
    }

    // Sum l over the 8 token lanes of each head column.
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }

    // ------------------------------------------- merge the 4 consumer warps --
    // The stage ring is idle now (every load was waited for); reuse it.
    float *red_m = reinterpret_cast<float *>(smem_gen);           // [4][8]
    float *red_l = red_m + kConsumerWarps * kHeadsPerCta;          // [4][8]
    float *red_o = red_l + kConsumerWarps * kHeadsPerCta;          // [4][8][HD]
    float *wts = red_o + kConsumerWarps * kHeadsPerCta * HD;       // [8][kMaxPartitions]
    float *wsum = wts + kHeadsPerCta * kMaxPartitions;             // [8]
    named_barrier_sync(1, kConsumerWarps * 32);
    if (g == 0) {
        red_m[warp * kHeadsPerCta + 2 * c] = m0;
        red_m[warp * kHeadsPerCta + 2 * c + 1] = m1;
        red_l[warp * kHeadsPerCta + 2 * c] = l0;
        red_l[warp * kHeadsPerCta + 2 * c + 1] = l1;
    }
#pragma unroll
    for (int i = 0; i < KSTEPS; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            red_o[(warp * kHeadsPerCta + 2 * c + (e & 1)) * HD + 16 * i + g + (e >> 1) * 8] = o[i][e];
    named_barrier_sync(1, kConsumerWarps * 32);

    const int ct = tid;  // 0..127
    const int64_t ws_row0 = ((int64_t)b * p.num_q_heads + head0) * gridDim.x;
    for (int idx = ct; idx < nh * HD; idx += kConsumerWarps * 32) {
        const int h = idx / HD, d = idx - (idx / HD) * HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red_m[w * kHeadsPerCta + h]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
            const float f = fast_exp2(red_m[w * kHeadsPerCta + h] - M);
            L += red_l[w * kHeadsPerCta + h] * f;
            O += red_o[(w * kHeadsPerCta + h) * HD + d] * f;
        }
        if (nparts == 1) {
            p.out[(int64_t)b * p.out_stride + (int64_t)(head0 + h) * HD + d] = __float2bfloat16(O / L);
        } else {
            const int64_t wr = ws_row0 + (int64_t)h * gridDim.x + part;
            p.ws_o[wr * HD + d] = O / L;
            if (d == 0) p.ws_lse[wr] = M + __log2f(L);
        }
    }
    if (nparts == 1) return;

    // ------------------------------------------------ split-K merge (last CTA) --
    __threadfence();
    named_barrier_sync(1, kConsumerWarps * 32);
    int *cnt = p.ws_cnt + (int64_t)b * gridDim.y + blockIdx.y;
    if (ct == 0) s_last = (atomicAdd(cnt, 1) == nparts - 1);
    named_barrier_sync(1, kConsumerWarps * 32);
    if (!s_last) return;
    __threadfence();
    for (int h = warp; h < nh; h += kConsumerWarps) {
        const float *lse = p.ws_lse + ws_row0 + (int64_t)h * gridDim.x;
        float M = -INFINITY;
        for (int q = lane; q < nparts; q += 32) M = fmaxf(M, __ldcg(lse + q));
        M = warp_max(M);
        float S = 0.f;
        for (int q = lane; q < nparts; q += 32) {
            const float w = fast_exp2(__ldcg(lse + q) - M);
            wts[h * kMaxPartitions + q] = w;
            S += w;
        }
        S = warp_sum(S);
        if (lane == 0) wsum[h] = S;
    }
    named_barrier_sync(1, kConsumerWarps * 32);
    for (int idx = ct; idx < nh * HD; idx += kConsumerWarps * 32) {
        const int h = idx / HD, d = idx - (idx / HD) * HD;
        const float *src = p.ws_o + (ws_row0 + (int64_t)h * gridDim.x) * HD + d;
        float acc = 0.f;
        for (int q = 0; q < nparts; ++q) acc += wts[h * kMaxPartitions + q] * __ldcg(src + (int64_t)q * HD);
        p.out[(int64_t)b * p.out_stride + (int64_t)(head0 + h) * HD + d] = __float2bfloat16(acc / wsum[h]);
    }
    if (ct == 0) *cnt = 0;  // leave the counter ready for the next call
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace layout of one call: counters [batch*Hq] int32 | lse [batch*Hq*parts]
// f32 | o [batch*Hq*parts*hd] f32. Counters sit first so that their place does
// not depend on the partition count.
size_t ws_counters_bytes(int batch, int hq) { return align256((size_t)batch * hq * 4); }
size_t ws_lse_bytes(int batch, int hq, int parts) { return align256((size_t)batch * hq * parts * 4); }
size_t ws_total(int batch, int hq, int hd, int parts) {
    return ws_counters_bytes(batch, hq) + ws_lse_bytes(batch, hq, parts) +
           (size_t)batch * hq * parts * hd * 4;
}

void choose_partitions(int batch, int hq, int hkv, int max_ctx, int partition_tokens, int *ptok,
                       int *parts) {
    if (max_ctx < 1) max_ctx = 1;
    int P;
    if (partition_tokens > 0) {
        P = (partition_tokens + kBlockSize - 1) / kBlockSize * kBlockSize;
    } else {
        const int group = hq / hkv;
        const int64_t units = (int64_t)batch * hkv * ((group + kHeadsPerCta - 1) / kHeadsPerCta);
        const int64_t target = 2 * (int64_t)sm_count();
        P = 512;
        while (P > 64 && units * ((max_ctx + P - 1) / P) < target) P >>= 1;
    }
    int n = (max_ctx + P - 1) / P;
    if (n > kMaxPartitions) n = kMaxPartitions;
    if (n < 1) n = 1;
    *ptok = P;
    *parts = n;
}


template <int HD>
int launch_decode(const DecodeParams &prm, int parts, int batch, const void *k_pool,
                  const void *v_pool, cudaStream_t stream) {
    CUtensorMap mk, mv;
    int rc = pool_tensor_map(k_pool, prm.pool_rows, HD, &mk);
    if (rc) return rc;
    rc = pool_tensor_map(v_pool, prm.pool_rows, HD, &mv);
    if (rc) return rc;
    const int smem = DecodeCfg<HD>::kSmemBytes;
    rc = ensure_smem_attr((const void *)paged_decode_kernel<HD>, smem);
    if (rc) return rc;
    dim3 grid(parts, prm.num_kv_heads * prm.ctas_per_kv, batch);
    paged_decode_kernel<HD><<<grid, kThreads, smem, stream>>>(mk, mv, prm);
    return launch_status();
}

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" size_t lc_paged_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                                 int head_dim, int max_partitions) {
    (void)num_kv_heads;
    if (batch <= 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
    if (max_partitions < 1) max_partitions = 1;
    if (max_partitions > kMaxPartitions) max_partitions = kMaxPartitions;
    return ws_total(batch, num_q_heads, head_dim, max_partitions);
}

extern "C" int lc_paged_decode_workspace_init(void *workspace, size_t workspace_bytes,
                                              lc_stream_t stream) {
    if (!workspace && workspace_bytes) return LC_ERR_INVALID_ARGUMENT;
    if (!workspace_bytes) return LC_OK;
    return cudaMemsetAsync(workspace, 0, workspace_bytes, as_stream(stream)) == cudaSuccess
               ? LC_OK
               : LC_ERR_CUDA;
}

extern "C" int lc_paged_decode_partitions(int batch, int num_q_heads, int num_kv_heads,
                                          int max_context_len, int partition_tokens) {
    if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0) return 1;
    int ptok, parts;
    choose_partitions(batch, num_q_heads, num_kv_heads, max_context_len, partition_tokens, &ptok,
                      &parts);
    return parts;
}

extern "C" int lc_paged_decode(void *out, int64_t out_stride, const void *q, int64_t q_stride,
                               const void *k_pool, const void *v_pool, int64_t num_blocks,
                               int num_layers, int layer, int num_q_heads, int num_kv_heads,
                               int head_dim, const int *block_tables, int table_stride,
                               const int *context_lens, int len_offset, int batch,
                               int max_context_len, int partition_tokens, float sm_scale,
                               void *workspace, size_t workspace_bytes, int *dev_status,
                               lc_stream_t stream) {
    if (!out || !q || !k_pool || !v_pool || !block_tables || !context_lens)
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (batch < 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || num_q_heads <= 0 ||
        num_kv_heads <= 0 || num_blocks <= 0 || table_stride <= 0 || len_offset < 0 ||
        len_offset > 1)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if (batch == 0) return LC_OK;
    if (batch > 65535) return LC_ERR_INVALID_ARGUMENT;
    if (!aligned16(k_pool) || !aligned16(v_pool) || !aligned16(q) || (q_stride & 7) ||
        ((uintptr_t)out & 1))
        return LC_ERR_MISALIGNED;
    if (q_stride < (int64_t)num_q_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim)
        return LC_ERR_INVALID_ARGUMENT;
    const int64_t pool_rows = num_blocks * num_layers * num_kv_heads * kBlockSize;
    if (pool_rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;

    int ptok, parts;
    choose_partitions(batch, num_q_heads, num_kv_heads, max_context_len, partition_tokens, &ptok,
                      &parts);
    DecodeParams prm{};
    prm.out = (bf16 *)out;
    prm.out_stride = out_stride;
    prm.q = (const bf16 *)q;
    prm.q_stride = q_stride;
    prm.tables = block_tables;
    prm.table_stride = table_stride;
    prm.ctx_lens = context_lens;
    prm.len_offset = len_offset;
    prm.pool_rows = pool_rows;
    prm.num_blocks = num_blocks;
    prm.num_layers = num_layers;
    prm.layer = layer;
    prm.num_q_heads = num_q_heads;
    prm.num_kv_heads = num_kv_heads;
    prm.group = num_q_heads / num_kv_heads;
    prm.ctas_per_kv = (prm.group + kHeadsPerCta - 1) / kHeadsPerCta;
    prm.partition_tokens = ptok;
    prm.scale_log2 = sm_scale * 1.4426950408889634f;
    prm.status = dev_status;
    if (parts > 1) {
        const size_t need = ws_total(batch, num_q_heads, head_dim, parts);
        if (!workspace || workspace_bytes < need || !aligned16(workspace))
            return workspace && !aligned16(workspace) ? LC_ERR_MISALIGNED
                                                      : LC_ERR_WORKSPACE_TOO_SMALL;
        uint8_t *ws = (uint8_t *)workspace;
        prm.ws_cnt = (int *)ws;
        prm.ws_lse = (float *)(ws + ws_counters_bytes(batch, num_q_heads));
        prm.ws_o = (float *)(ws + ws_counters_bytes(batch, num_q_heads) +
                             ws_lse_bytes(batch, num_q_heads, parts));
    }
    cudaStream_t s = as_stream(stream);
    return head_dim == 64 ? launch_decode<64>(prm, parts, batch, k_pool, v_pool, s)
                          : launch_decode<128>(prm, parts, batch, k_pool, v_pool, s);
}

extern "C" size_t lc_flash_decoding_workspace_size(int num_q_heads, int head_dim,
                                                   int max_seq_len) {
    int parts = (max_seq_len + 63) / 64;
    return lc_paged_decode_workspace_size(1, num_q_heads, 1, head_dim, parts);
}

extern "C" int lc_flash_decoding(void *output, const void *q, const void *k_pool,
                                 const void *v_pool, const int *block_table, int layer_idx,
                                 int num_q_heads, int num_kv_heads, int head_dim,
                                 int max_seq_len, const int *current_pos, float sm_scale,
                                 int block_size, int num_layers, int host_pos,
                                 int64_t num_physical_blocks, void *workspace,
                                 size_t workspace_bytes, lc_stream_t stream) {
    if (block_size != kBlockSize) return LC_ERR_UNSUPPORTED_SHAPE;
    if (host_pos < 0 || max_seq_len <= 0) return LC_ERR_INVALID_ARGUMENT;
    // The reference's table holds ceil(max_position_embeddings / 16) entries
    // (src/layers/kv_cache.rs:70-71).
    int table_len = (max_seq_len + kBlockSize - 1) / kBlockSize;
    if (table_len < host_pos / kBlockSize + 1) table_len = host_pos / kBlockSize + 1;
    const int64_t stride = (int64_t)num_q_heads * head_dim;
    return lc_paged_decode(output, stride, q, stride, k_pool, v_pool, num_physical_blocks,
                           num_layers, layer_idx, num_q_heads, num_kv_heads, head_dim,
                           block_table, table_len, current_pos, /*len_offset=*/1, 1,
                           host_pos + 1, 0, sm_scale, workspace, workspace_bytes, nullptr,
                           stream);
}
