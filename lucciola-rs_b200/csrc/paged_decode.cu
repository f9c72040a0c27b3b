// paged_decode.cu - batched paged flash-decoding attention for GQA (sm_100a).
//
// Replaces flash_decoding_kernel_64/128 (src/kernels/attention.cu:4-240), which
// runs one 1024-thread CTA per query head over one sequence and so reads every
// KV byte Hq/Hkv times with scalar 2-byte loads. Here:
//
//  * Work unit = one 16-token page of one (sequence, kv head [8-head slice])
//    "segment"; a CTA serves all query heads of the kv head's group (up to 8),
//    so each KV byte leaves HBM once.
//  * Persistent, balanced grid: the pages of all segments form one global
//    stream (segment order b-major, then kv head); CTA c of C takes the
//    contiguous range [c*T/C, (c+1)*T/C) of the T pages, crossing segment
//    boundaries. Every CTA moves the same number of bytes whatever the context
//    lengths are, and its pipeline never drains between segments.
//  * A producer warp streams the range into a ring of shared-memory stages
//    with TMA tile loads (one {64 x 16} box per half page, 128-byte swizzle);
//    the first stage of every chunk also carries the chunk's query rows (bulk
//    copy). mbarriers with transaction counts track completion.
//  * Four consumer warps each take one page per stage and run both products on
//    the tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate) with tokens
//    on M and the <= 8 query heads on N:
//        S^T[16 tok x 8 heads]  = K_page[16 x hd] . Q^T[hd x 8]
//        O^T[hd x 8 heads]     += V_page^T[hd x 16] . P^T[16 x 8]
//    P^T moves from the accumulator layout to the B-operand layout with
//    movmatrix.trans. Online softmax in base 2.
//  * A chunk that covers a whole segment writes the bf16 output directly. A
//    segment split across CTAs writes (O/l, log2-sum-exp) partials as tagged
//    words; the last CTA to finish it (arrival counter) merges them in slot
//    order from its stage ring.
//  * One sequence (the fused entry with batch 1): each segment's pages go to
//    one thread-block cluster instead, and the pieces are sent into rank 0's
//    shared memory with st.async, their bytes counted on rank 0's mbarrier;
//    rank 0 combines them in rank order (no workspace, no counter).
//
// Semantics follow attention.cu: out = softmax(q.k * scale) . v over cache
// tokens 0..n-1, fp32 accumulation, bf16 output. Block-table entries outside
// the pool are reported in the status word and read as zeros (TMA bounds fill).
#include <climits>
#include <mutex>

#include "lc_common.cuh"
#include "lc_host.h"
#include "rope_math.cuh"

namespace lc {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kProducerWarp = kConsumerWarps;      // warp 4
constexpr int kEpilogueWarp = kConsumerWarps + 1;  // warp 5
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr int kHeadsPerCta = 8;
constexpr int kPagesPerStage = kConsumerWarps;  // one page per consumer warp per stage
constexpr int kMaxPeers = LC_PEER_MAX_RANKS - 1;
constexpr int kMinPagesPerCta = 8;               // auto split: two stages per CTA at least
// Single-sequence path: the pages of each segment are split over one thread-
// block cluster, whose rank 0 gathers the pieces in its shared memory.
constexpr int kClusterMax = 16;
#ifndef LC_CL_MIN_PAGES
#define LC_CL_MIN_PAGES 4
#endif
constexpr int kClusterMinPages = LC_CL_MIN_PAGES;  // pages per CTA at least

// kFinal marks the last stage of the CTA's whole range.
enum : int { kFirst = 1, kLast = 2, kDone = 4, kFinal = 8 };

struct StageMeta {
    int b, g, page0, np;    // sequence, segment-in-sequence, first page of the stage, pages
    int n, pages_b, flags;  // tokens of the sequence, its pages, kFirst/kLast/kDone/kFinal
    int chunk_p0, take;     // chunk = pages [chunk_p0, chunk_p0 + take) of the segment
    int pos;                // fused: the new token's position (unclamped)
    long long seg_start;    // global index of the segment's first page
};

// Finished chunk handed from the consumer warps to the epilogue warp.
struct EpiInfo {
    int b, seg, nh, head0, pages_b, whole, done;
    long long seg_start;
};

template <int HD>
struct DecodeCfg {
    static constexpr int kPageBytes = kBlockSize * HD * 2;  // 2 KiB / 4 KiB
    static constexpr int kStages = HD == 64 ? 4 : 3;
    static constexpr int kStageBytes = kPagesPerStage * 2 * kPageBytes;  // K pages, V pages
    static constexpr int kQBytes = kHeadsPerCta * HD * 2;
    static constexpr int kRedFloats = kHeadsPerCta * HD + 2 * kHeadsPerCta;  // o, m, l
    static constexpr int kQOffset = kStages * kStageBytes;
    static constexpr int kRedOffset = kQOffset + kStages * kQBytes;
    static constexpr int kSmemBytes = kRedOffset + 2 * kRedFloats * 4 + 1024;  // + alignment
    // Cluster path: one slot per CTA of the cluster in rank 0, [8][HD] fp32
    // normalised partial then [8] fp32 log2-sum-exp.
    static constexpr int kClSlotFloats = kHeadsPerCta * HD + kHeadsPerCta;
    static constexpr int kClOffset = kRedOffset + 2 * kRedFloats * 4;
    static constexpr int kRed4Offset = kClOffset + kClusterMax * kClSlotFloats * 4;
    static constexpr int kSmemClusterBytes = kRed4Offset + 2 * kRedFloats * 4 + 1024;
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
    int batch;
    int64_t pool_rows;  // rows of the [rows][hd] pool view; used as an all-out-of-bounds row
    int64_t num_blocks;
    int num_layers, layer, num_q_heads, num_kv_heads, group, ctas_per_kv;
    int seg_per_seq;  // num_kv_heads * ctas_per_kv
    int partition_tokens;
    float scale_log2;  // sm_scale * log2(e)
    // Programmatic dependent launch (lc_set_dependent_launch): 1 = every warp
    // waits for the preceding grid first; 2 = set-up (context lengths, split)
    // runs before that wait, and in the fused kernel the producer warp, which
    // only reads context lengths, block tables and this layer's cached pages,
    // never waits: its first stages land while the preceding grid drains; the
    // epilogue warp reads the first chunk's position, rope rows and biases
    // before it and only the qkv rows after.
    int pdl_mode;
    // out and out_stride keep bf16 pairs 4-byte aligned (else element stores).
    int out_vec;
    uint64_t *ws_o;    // [slots][8][HD] tagged words (split-segment partials)
    uint64_t *ws_lse;  // [slots][8] tagged words
    int *ws_cnt;       // [batch * seg_per_seq]
    int *status;
    // Fused bias + RoPE + append (FUSED kernels only). q/q_stride then address
    // qkv rows [q | k | v]; context_lens holds the new token's position.
    const bf16 *qkv;
    const bf16 *q_bias, *k_bias, *v_bias;
    // Optional input gate: the qkv rows are read only once *gate != 0 (a flag
    // a copy stream sets after the rows' host-to-device copy).
    const int *gate;
    const float *cos_t, *sin_t;
    int rope_rows;
    bf16 *k_pool_w, *v_pool_w;
    // Peer exchange (PEER kernels only): every output row is also stored at
    // its address + peer_delta[r], r < n_peer (the same row of a peer's output
    // buffer, mapped into this process). After its last store each CTA counts
    // itself on peer_done; the grid's last CTA resets it, advances peer_seq and
    // stores the new count into every peer_flag[r] (system-scope release).
    int n_peer;
    long long peer_delta[kMaxPeers];
    int *peer_flag[kMaxPeers];
    int *peer_done, *peer_seq;
};

// Shared-memory byte address of 16-byte chunk `kc` (of hd/8) of token row `r` in a
// page tile stored as hd/64 boxes of [16 rows][128 B] with 128-byte swizzle.
__device__ __forceinline__ uint32_t tile_addr(uint32_t page, int r, int kc) {
    return page + ((kc >> 3) << 11) + (r << 7) + ((((kc & 7) ^ (r & 7))) << 4);
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void fence_acq_rel_sys() {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// An output element; PEER kernels store it into every peer's buffer as well.
template <bool PEER>
__device__ __forceinline__ void put_out(const DecodeParams &p, bf16 *a, bf16 v) {
    *a = v;
    if constexpr (PEER) {
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r)
            if (r < p.n_peer)
                *reinterpret_cast<bf16 *>(reinterpret_cast<char *>(a) + p.peer_delta[r]) = v;
    }
}

// PEER kernels: one thread per CTA, once every output store of the CTA has
// been fenced at system scope by the thread that made it and a barrier has
// joined them. The wait for the preceding grid comes first, so that a CTA of
// a launch that started early (programmatic dependent launch) never counts
// while the previous launch's CTAs still do. The grid's last CTA publishes.
__device__ __forceinline__ void peer_arrive(const DecodeParams &p) {
    griddep_wait();
    if (atomicAdd(p.peer_done, 1) != (int)gridDim.x - 1) return;
    fence_acq_rel_sys();  // acquire side of the other CTAs' fence + count
    *p.peer_done = 0;     // ready for the next launch
    const int seq = *p.peer_seq + 1;
    *p.peer_seq = seq;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
        if (r < p.n_peer)
            asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p.peer_flag[r]), "r"(seq)
                         : "memory");
}


__device__ __forceinline__ int seq_tokens(const DecodeParams &p, int b, bool report) {
    int n = __ldg(p.ctx_lens + b) + p.len_offset;
    if (n < 0) n = 0;
    const int cap = p.table_stride * kBlockSize;
    if (n > cap) {
        if (report) set_status(p.status, LC_DEV_BAD_POS);
        n = cap;
    }
    return n;
}

// One chunk: the pages [p0, p0 + take) of segment g of sequence b that a CTA's
// range covers.
struct Chunk {
    int b, g, p0, take, n, pages_b;
    long long seg_start;  // global index of the segment's first page
};

// Walks the chunks of the range [start, end) of the global page stream in
// order. The producer warp and, in the fused kernel, the epilogue warp each run
// one, so both see the same chunk sequence.
struct ChunkCursor {
    int b, g, pg, n, pages_b;
    long long glob;

    __device__ __forceinline__ void init(const DecodeParams &p, long long start, int b0,
                                         long long pref_b0, bool report) {
        b = b0;
        n = seq_tokens(p, b, report);
        pages_b = (n + kBlockSize - 1) / kBlockSize;  // > 0: b0 holds page `start`
        const long long off = start - pref_b0;
        g = (int)(off / pages_b);
        pg = (int)(off - (long long)g * pages_b);
        glob = start;
    }

    __device__ __forceinline__ bool next(const DecodeParams &p, long long end, bool report,
                                         Chunk &c) {
        while (glob < end) {
            if (pages_b == 0) {  // empty sequence: owns no pages
                ++b;
                n = seq_tokens(p, b, report);
                pages_b = (n + kBlockSize - 1) / kBlockSize;
                continue;
            }
            c.b = b;
            c.g = g;
            c.p0 = pg;
            c.n = n;
            c.pages_b = pages_b;
            c.take = (int)min((long long)(pages_b - pg), end - glob);
            c.seg_start = glob - pg;
            glob += c.take;
            pg = 0;
            if (++g == p.seg_per_seq) {
                g = 0;
                ++b;
                if (glob < end) {
                    n = seq_tokens(p, b, report);
                    pages_b = (n + kBlockSize - 1) / kBlockSize;
                }
            }
            return true;
        }
        return false;
    }
};

// Fused mode, epilogue warp: waits (bounded) until *gate is non-zero before
// the first qkv row is read. Lane 0 polls with acquire loads; a timeout sets
// LC_DEV_TIMEOUT and the abort flag (the rows are then not trusted).
__device__ __forceinline__ void gate_wait(const int *gate, volatile int *abort_flag, int *status,
                                          int lane) {
    if (lane == 0) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(gate) : "memory");
        if (v == 0) {
            const uint64_t t0 = global_timer_ns();
            for (uint32_t it = 1;; ++it) {
                asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(gate) : "memory");
                if (v != 0) break;
                if ((it & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
                    *abort_flag = 1;
                    set_status(status, LC_DEV_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncwarp();
}

// Fused mode, epilogue warp: everything a chunk needs from the qkv rows, made
// ahead of the consumer warps (signalled on `ready`):
//  * q of the chunk's <= 8 query heads, bias added and rotated, bf16 [8][HD]
//    in `qs` (zeros for heads past the group);
//  * when the chunk ends with the sequence's new token: its rotated K row and
//    V + bias row, bf16 [2][HD] in `nk`, which the consumer warp holding that
//    page writes over the tile row; the first 8-head slice of the kv head also
//    appends both rows to the pools here.
// load_static() reads what no preceding kernel of a decode step writes (the
// position, rope rows, biases, block table), so for the first chunk it runs
// before the programmatic-dependency wait; finish() reads the qkv row. The
// arithmetic is that of rope_append.cu (rope_math.cuh), so q, the tile rows and
// the pool writes equal the two-launch path's bit for bit.
template <int HD>
struct ChunkPrep {
    static constexpr int kHalf = HD / 2;
    static constexpr int kPer = kHalf / 4;  // q dims per lane (lane: head lane / 4, quarter lane % 4)
    static constexpr int kNk = HD / 64;     // new-token rotation pairs per lane
    int pos, head0, nh, kvh, hsub, phys;
    bool pos_ok, has_nk;
    float2 cs[kPer / 2], sv[kPer / 2];
    __nv_bfloat162 b1[kPer / 2], b2[kPer / 2];
    float kc[kNk], ks[kNk];
    bf16 kb1[kNk], kb2[kNk], vb1[kNk], vb2[kNk];

    __device__ __forceinline__ void load_static(const DecodeParams &p, const Chunk &c, int lane) {
        kvh = c.g / p.ctas_per_kv;
        hsub = c.g - kvh * p.ctas_per_kv;
        head0 = kvh * p.group + hsub * kHeadsPerCta;
        nh = min(kHeadsPerCta, p.group - hsub * kHeadsPerCta);
        pos = __ldg(p.ctx_lens + c.b) + p.len_offset - 1;
        pos_ok = pos >= 0 && pos < p.rope_rows;
        const float *ct = p.cos_t + (int64_t)(pos_ok ? pos : 0) * kHalf;
        const float *sn = p.sin_t + (int64_t)(pos_ok ? pos : 0) * kHalf;
        const int h = lane >> 2, d0 = (lane & 3) * kPer;
        const bf16 *bias = p.q_bias + (int64_t)(head0 + min(h, nh - 1)) * HD;
#pragma unroll
        for (int i = 0; i < kPer / 2; ++i) {
            const int d = d0 + 2 * i;
            b1[i] = __ldg(reinterpret_cast<const __nv_bfloat162 *>(bias + d));
            b2[i] = __ldg(reinterpret_cast<const __nv_bfloat162 *>(bias + d + kHalf));
            cs[i] = pos_ok ? __ldg(reinterpret_cast<const float2 *>(ct + d)) : make_float2(1.f, 1.f);
            sv[i] = pos_ok ? __ldg(reinterpret_cast<const float2 *>(sn + d)) : make_float2(0.f, 0.f);
        }
        has_nk = pos == c.n - 1 && c.p0 + c.take == c.pages_b;
        if (has_nk) {
            phys = __ldg(p.tables + (int64_t)c.b * p.table_stride + c.pages_b - 1);
#pragma unroll
            for (int i = 0; i < kNk; ++i) {
                const int d = lane + 32 * i;
                kb1[i] = p.k_bias[kvh * HD + d];
                kb2[i] = p.k_bias[kvh * HD + d + kHalf];
                vb1[i] = p.v_bias[kvh * HD + d];
                vb2[i] = p.v_bias[kvh * HD + d + kHalf];
                kc[i] = pos_ok ? __ldg(ct + d) : 1.f;
                ks[i] = pos_ok ? __ldg(sn + d) : 0.f;
            }
        }
    }

    __device__ __forceinline__ void finish(const DecodeParams &p, const Chunk &c, bf16 *qs, bf16 *nk,
                                           uint64_t *ready, int lane) const {
        const bf16 *qkv_row = p.qkv + (int64_t)c.b * p.q_stride;
        const int h = lane >> 2, d0 = (lane & 3) * kPer;
        bf16 *dst = qs + h * HD;
        if (h < nh) {
            const bf16 *row = qkv_row + (int64_t)(head0 + h) * HD;
#pragma unroll
            for (int i = 0; i < kPer / 2; ++i) {
                const int d = d0 + 2 * i;
                const __nv_bfloat162 x1 = *reinterpret_cast<const __nv_bfloat162 *>(row + d);
                const __nv_bfloat162 x2 = *reinterpret_cast<const __nv_bfloat162 *>(row + d + kHalf);
                const float a0 = __fadd_rn(__low2float(x1), __low2float(b1[i]));
                const float a1 = __fadd_rn(__high2float(x1), __high2float(b1[i]));
                const float e0 = __fadd_rn(__low2float(x2), __low2float(b2[i]));
                const float e1 = __fadd_rn(__high2float(x2), __high2float(b2[i]));
                *reinterpret_cast<__nv_bfloat162 *>(dst + d) =
                    __halves2bfloat162(__float2bfloat16(rot_sub(a0, cs[i].x, e0, sv[i].x)),
                                       __float2bfloat16(rot_sub(a1, cs[i].y, e1, sv[i].y)));
                *reinterpret_cast<__nv_bfloat162 *>(dst + d + kHalf) =
                    __halves2bfloat162(__float2bfloat16(rot_add(a0, sv[i].x, e0, cs[i].x)),
                                       __float2bfloat16(rot_add(a1, sv[i].y, e1, cs[i].y)));
            }
        } else {
            const __nv_bfloat162 z = __float2bfloat162_rn(0.f);
#pragma unroll
            for (int i = 0; i < kPer; i += 2) {
                *reinterpret_cast<__nv_bfloat162 *>(dst + d0 + i) = z;
                *reinterpret_cast<__nv_bfloat162 *>(dst + d0 + i + kHalf) = z;
            }
        }
        if (has_nk) {
            const int ko = p.num_q_heads * HD + kvh * HD, vo = ko + p.num_kv_heads * HD;
            const bool append = hsub == 0;
            const bool ph_ok = phys >= 0 && phys < p.num_blocks;
            const int64_t prow =
                page_row(ph_ok ? phys : 0, p.layer, kvh, p.num_layers, p.num_kv_heads) * HD +
                (int64_t)(pos % kBlockSize) * HD;
#pragma unroll
            for (int i = 0; i < kNk; ++i) {
                const int d = lane + 32 * i;
                const float a1 = __fadd_rn(__bfloat162float(qkv_row[ko + d]), __bfloat162float(kb1[i]));
                const float a2 = __fadd_rn(__bfloat162float(qkv_row[ko + d + kHalf]), __bfloat162float(kb2[i]));
                const bf16 rk1 = __float2bfloat16(rot_sub(a1, kc[i], a2, ks[i]));
                const bf16 rk2 = __float2bfloat16(rot_add(a1, ks[i], a2, kc[i]));
                const bf16 rv1 = __float2bfloat16(__fadd_rn(__bfloat162float(qkv_row[vo + d]), __bfloat162float(vb1[i])));
                const bf16 rv2 = __float2bfloat16(__fadd_rn(__bfloat162float(qkv_row[vo + d + kHalf]), __bfloat162float(vb2[i])));
                nk[d] = rk1;
                nk[d + kHalf] = rk2;
                nk[HD + d] = rv1;
                nk[HD + d + kHalf] = rv2;
                if (append && ph_ok) {
                    p.k_pool_w[prow + d] = rk1;
                    p.k_pool_w[prow + d + kHalf] = rk2;
                    p.v_pool_w[prow + d] = rv1;
                    p.v_pool_w[prow + d + kHalf] = rv2;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(ready);
    }
};

// Fused mode, consumer warp: the new token's K and V rows (bf16 [2][HD] at
// `nk`) over row r of the page tiles. Lane l copies 16-byte chunk l of each.
template <int HD>
__device__ __forceinline__ void patch_new_row(const bf16 *nk, uint8_t *smem_gen, uint32_t smem_base,
                                              uint32_t kpage, uint32_t vpage, int r, int lane) {
    constexpr int kChunks = HD / 8;
    if (lane < kChunks) {
        const uint4 kv = reinterpret_cast<const uint4 *>(nk)[lane];
        const uint4 vv = reinterpret_cast<const uint4 *>(nk + HD)[lane];
        *reinterpret_cast<uint4 *>(smem_gen + (tile_addr(kpage, r, lane) - smem_base)) = kv;
        *reinterpret_cast<uint4 *>(smem_gen + (tile_addr(vpage, r, lane) - smem_base)) = vv;
    }
}

// Sequences without cached tokens own no pages: their output rows are zero.
// CTA `first` of `count` zeroes sequences first, first + count, ...
template <int HD, bool PEER>
__device__ __forceinline__ void zero_empty_outputs(const DecodeParams &p, int first, int count,
                                                   int t, int nthreads) {
    for (int b = first; b < p.batch; b += count)
        if (seq_tokens(p, b, false) == 0)
            for (int i = t; i < p.num_q_heads * HD; i += nthreads)
                put_out<PEER>(p, p.out + (int64_t)b * p.out_stride + i, __float2bfloat16(0.f));
}

// Owner CTA of global page x under the balanced split start(c) = c*T/C.
__device__ __forceinline__ int owner_cta(long long x, long long T, int C) {
    return (int)(((x + 1) * C - 1) / T);
}

__device__ __forceinline__ void bulk_load(void *smem_dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Barrier of the 128 consumer threads built on an mbarrier, so that a warp
// that gave up on a wait cannot leave the others blocked for good.
__device__ __forceinline__ bool consumer_sync(uint64_t *bar, uint32_t &phase,
                                              volatile int *abort_flag, int *status) {
    // One arrival per warp: 128 arrivals on one barrier word queue up behind
    // each other in the shared-memory unit.
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    const bool ok = mbar_wait_bounded(bar, phase & 1, abort_flag, status);
    ++phase;
    return ok;
}

// ------------------------------------------------ thread-block cluster path --
__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cl_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of `local` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t cl_map(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ void cl_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
// Stores into another CTA's shared memory that count their bytes, on landing,
// against that CTA's mbarrier (complete_tx): no fence and no separate arrival.
__device__ __forceinline__ void st_async_f32(uint32_t a, float v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(a),
                 "f"(v), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void st_async_f32x2(uint32_t a, float x, float y, uint32_t bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(a),
        "f"(x), "f"(y), "r"(bar)
        : "memory");
}

// Per-warp running softmax state of one chunk: heads 2c, 2c+1 of this lane.
template <int HD>
struct WarpState {
    float o[HD / 16][4];
    float m0, m1, l0, l1;
    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int i = 0; i < HD / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
    }
};

// red slot layout: o[8][HD], m[8], l[8] (floats)
template <int HD>
__device__ __forceinline__ void state_store(float *red, const WarpState<HD> &st, int lane) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int i = 0; i < HD / 16; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            red[(2 * c + (e & 1)) * HD + 16 * i + g + (e >> 1) * 8] = st.o[i][e];
    if (g == 0) {
        red[kHeadsPerCta * HD + 2 * c] = st.m0;
        red[kHeadsPerCta * HD + 2 * c + 1] = st.m1;
        red[kHeadsPerCta * HD + kHeadsPerCta + 2 * c] = st.l0;
        red[kHeadsPerCta * HD + kHeadsPerCta + 2 * c + 1] = st.l1;
    }
}

template <int HD>
__device__ __forceinline__ void state_combine(WarpState<HD> &st, const float *red, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const float om0 = red[kHeadsPerCta * HD + 2 * c], om1 = red[kHeadsPerCta * HD + 2 * c + 1];
    const float ol0 = red[kHeadsPerCta * HD + kHeadsPerCta + 2 * c];
    const float ol1 = red[kHeadsPerCta * HD + kHeadsPerCta + 2 * c + 1];
    const float M0 = fmaxf(st.m0, om0), M1 = fmaxf(st.m1, om1);
    const float u0 = M0 == -INFINITY ? 0.f : M0, u1 = M1 == -INFINITY ? 0.f : M1;
    const float a0 = fast_exp2(st.m0 - u0), b0 = fast_exp2(om0 - u0);
    const float a1 = fast_exp2(st.m1 - u1), b1 = fast_exp2(om1 - u1);
    st.m0 = M0;
    st.m1 = M1;
    st.l0 = st.l0 * a0 + ol0 * b0;
    st.l1 = st.l1 * a1 + ol1 * b1;
#pragma unroll
    for (int i = 0; i < HD / 16; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float other = red[(2 * c + (e & 1)) * HD + 16 * i + g + (e >> 1) * 8];
            st.o[i][e] = (e & 1) ? st.o[i][e] * a1 + other * b1 : st.o[i][e] * a0 + other * b0;
        }
}

// ---- split segments ---------------------------------------------------------
// A segment whose pages span several CTAs ("pieces") is finished by the last
// piece to arrive on the segment's counter. Every other piece leaves its
// normalised result (O/l per head and dim, and log2-sum-exp per head) in its
// workspace slot as 64-bit words: the value's bits low, a tag (1) high. A word
// is written and read whole (single-copy atomic), so the merger sees either an
// old cleared word (tag 0) or the new value, and needs no fence from the
// writer: it re-reads a word until its tag is set (bounded). The merger clears
// every word it consumed, so all tags are 0 again when the launch ends.
constexpr uint64_t kPartTag = 1ull << 32;

__device__ __forceinline__ uint64_t part_word(float v) { return kPartTag | __float_as_uint(v); }

// Plain stores: an aligned 8-byte store is written whole; strong (relaxed.gpu)
// stores cost several times more issue time here for no gain, as the reader
// re-checks every word's tag.
__device__ __forceinline__ void st_part(uint64_t *a, uint64_t x) {
    asm volatile("st.global.b64 [%0], %1;" ::"l"(a), "l"(x) : "memory");
}
__device__ __forceinline__ void st_part2(uint64_t *a, uint64_t x, uint64_t y) {
    asm volatile("st.global.v2.b64 [%0], {%1, %2};" ::"l"(a), "l"(x), "l"(y) : "memory");
}
__device__ __forceinline__ uint64_t ld_part(const uint64_t *a) {
    uint64_t x;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(x) : "l"(a) : "memory");
    return x;
}
__device__ __forceinline__ void ld_part2(const uint64_t *a, uint64_t &x, uint64_t &y) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(a)
                 : "memory");
}

// Running log-sum-exp combination of normalised partials (base 2): the result
// is acc / s; m is the largest log2-sum-exp combined so far.
template <int ND>
struct LseAcc {
    float acc[ND];
    float m, s;
    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int i = 0; i < ND; ++i) acc[i] = 0.f;
        m = -INFINITY;
        s = 0.f;
    }
    __device__ __forceinline__ void add(const float (&o)[ND], float lse) {
        const float mn = fmaxf(m, lse);  // finite: a piece holds at least one token
        const float a = fast_exp2(m - mn), b = fast_exp2(lse - mn);
#pragma unroll
        for (int i = 0; i < ND; ++i) acc[i] = acc[i] * a + o[i] * b;
        s = s * a + b;
        m = mn;
    }
};

// bf16 pairs of one head's output: pair k at dims 32k + 2t, 32k + 2t + 1
// (NP = HD / 32 pairs); PEER kernels store them into every peer's buffer too.
template <int NP, bool PEER>
__device__ __forceinline__ void put_out_pairs(const DecodeParams &p, bf16 *head_row, int t,
                                              const float (&v)[2 * NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        bf16 *a = head_row + 32 * k + 2 * t;
        if (!p.out_vec) {  // rows not 4-byte aligned: element stores
            put_out<PEER>(p, a, __float2bfloat16(v[2 * k]));
            put_out<PEER>(p, a + 1, __float2bfloat16(v[2 * k + 1]));
            continue;
        }
        const uint32_t w = pack_bf16(v[2 * k], v[2 * k + 1]);
        *reinterpret_cast<uint32_t *>(a) = w;
        if constexpr (PEER) {
#pragma unroll
            for (int r = 0; r < kMaxPeers; ++r)
                if (r < p.n_peer)
                    *reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(a) + p.peer_delta[r]) = w;
        }
    }
}

// Consumer-thread share of a segment's [8][HD] result in the final-chunk path:
// thread ct (0..127) owns head h = ct >> 4 and, with t = ct & 15, the dim
// pairs 32k + 2t (+1), k < HD / 32. Sixteen threads of a head thus read and
// write 16 consecutive pairs at a time (no shared-memory bank conflicts).
template <int HD>
struct ShareMap {
    static constexpr int NP = HD / 32;  // pairs per thread
    static constexpr int ND = 2 * NP;   // values per thread
    int h, t;
    __device__ __forceinline__ explicit ShareMap(int ct) : h(ct >> 4), t(ct & 15) {}
    __device__ __forceinline__ int dim(int k) const { return 32 * k + 2 * t; }
};

// Cluster path: consumer thread ct's share of this CTA's piece (its head's dim
// pairs, and the log2-sum-exp when t == 0) into slot `rank` of rank 0's gather
// buffer. Every rank's 128 threads each send their share exactly once, so rank
// 0's barrier completes when kClSlotFloats * 4 bytes per rank have landed.
template <int HD>
__device__ __forceinline__ void cl_send(int ct, const float (&o)[HD / 16], float lse,
                                        uint32_t buf_local, uint64_t *bar) {
    const ShareMap<HD> sm(ct);
    const uint32_t rb = cl_map(smem_u32(bar), 0);
    const uint32_t slot = cl_map(buf_local, 0) + cl_rank() * DecodeCfg<HD>::kClSlotFloats * 4;
#pragma unroll
    for (int k = 0; k < ShareMap<HD>::NP; ++k)
        st_async_f32x2(slot + (uint32_t)(sm.h * HD + sm.dim(k)) * 4, o[2 * k], o[2 * k + 1], rb);
    if (sm.t == 0) st_async_f32(slot + (uint32_t)(kHeadsPerCta * HD + sm.h) * 4, lse, rb);
}
template <int HD>
__device__ __forceinline__ void cl_send_empty(int ct, uint32_t buf_local, uint64_t *bar) {
    const float z[HD / 16] = {};
    cl_send<HD>(ct, z, -INFINITY, buf_local, bar);
}

// Merge of split segment `seg` by its last piece, run by the 128 consumer
// threads once the stage ring is idle: pieces j = 0..nch-1 sit in slots
// slot0 + j; piece `own` (or none, -1) is this CTA's, whose normalised result
// and log2-sum-exp the caller holds (`own_o`, `own_lse`; its words are in its
// slot too). The slots' words come into the ring with one bulk copy per batch
// (all of the segment's pieces in one round trip when they fit); a thread that
// finds one of its words still untagged (the piece's stores are on their way)
// reads those words again from global memory until they are (bounded). Pieces
// are combined in slot order, the same whichever piece merges, so the result
// does not depend on arrival order. Writes the head's outputs to `orow` (null:
// the head is past the group) and clears every consumed word. Returns false
// when a wait gave up (abort flag and status set).
template <int HD, bool PEER>
__device__ __forceinline__ bool merge_split_segment(
    const DecodeParams &p, long long slot0, int nch, int own, const float (&own_o)[HD / 16],
    float own_lse, const ShareMap<HD> &sm, bf16 *orow, uint8_t *ring, uint64_t *bar,
    uint32_t &bar_phase, uint64_t *sync_bar, uint32_t &sync_phase, volatile int *abort_flag,
    bool leader) {
    constexpr int NP = ShareMap<HD>::NP, ND = ShareMap<HD>::ND;
    constexpr int kPartWords = kHeadsPerCta * HD;
    constexpr int kRingBytes = DecodeCfg<HD>::kStages * DecodeCfg<HD>::kStageBytes;
    constexpr int kMax = kRingBytes / ((kPartWords + kHeadsPerCta) * 8);
    static_assert(kMax >= 8, "the ring holds at least 8 pieces");
    const int h = sm.h;
    const uint64_t *ro = reinterpret_cast<const uint64_t *>(ring);
    const uint64_t *rl = ro + kMax * kPartWords;
    LseAcc<ND> acc;
    acc.reset();
    for (int j0 = 0; j0 < nch; j0 += kMax) {
        const int cnt = min(kMax, nch - j0);
        if (j0 > 0 && !consumer_sync(sync_bar, sync_phase, abort_flag, p.status))
            return false;  // every thread is done with the previous batch
        if (leader) {
            // Words written by other CTAs (generic proxy) and the ring's last
            // generic reads, before the bulk copy (async proxy).
            asm volatile("fence.proxy.async.global;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const uint32_t ob = (uint32_t)(cnt * kPartWords * 8), lb = (uint32_t)(cnt * kHeadsPerCta * 8);
            mbar_arrive_expect_tx(bar, ob + lb);
            bulk_load(ring, p.ws_o + (slot0 + j0) * kPartWords, ob, bar);
            bulk_load(const_cast<uint64_t *>(rl), p.ws_lse + (slot0 + j0) * kHeadsPerCta, lb, bar);
        }
        if (!mbar_wait_bounded(bar, bar_phase & 1, abort_flag, p.status)) {
            if (leader) mbar_wait_drain(bar, bar_phase & 1);
            return false;
        }
        ++bar_phase;
        for (int jj = 0; jj < cnt; ++jj) {
            const int j = j0 + jj;
            if (j == own) {
                acc.add(own_o, own_lse);
                continue;
            }
            // Value bits low, tag high: x/z values, y/w tags of the two words.
            uint2 lw = *reinterpret_cast<const uint2 *>(rl + jj * kHeadsPerCta + h);
            uint4 q[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k)
                q[k] = *reinterpret_cast<const uint4 *>(ro + jj * kPartWords + h * HD + sm.dim(k));
            auto all_tagged = [&]() {
                uint32_t ok = lw.y == 1u;
#pragma unroll
                for (int k = 0; k < NP; ++k) ok &= (q[k].y == 1u) & (q[k].w == 1u);
                return ok != 0;
            };
            if (!all_tagged()) {  // a store of that piece had not landed when copied
                const long long slot = slot0 + j;
                const uint64_t *src = p.ws_o + (slot * kHeadsPerCta + h) * HD;
                const uint64_t t0 = global_timer_ns();
                for (uint32_t it = 1; !all_tagged(); ++it) {
                    if ((it & 63u) == 0 && (*abort_flag || global_timer_ns() - t0 > kWaitLimitNs)) {
                        *abort_flag = 1;
                        set_status(p.status, LC_DEV_TIMEOUT);
                        return false;
                    }
                    const uint64_t l64 = ld_part(p.ws_lse + slot * kHeadsPerCta + h);
                    lw = make_uint2((uint32_t)l64, (uint32_t)(l64 >> 32));
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        uint64_t a, b;
                        ld_part2(src + sm.dim(k), a, b);
                        q[k] = make_uint4((uint32_t)a, (uint32_t)(a >> 32), (uint32_t)b, (uint32_t)(b >> 32));
                    }
                }
            }
            float v[ND];
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                v[2 * k] = __uint_as_float(q[k].x);
                v[2 * k + 1] = __uint_as_float(q[k].z);
            }
            acc.add(v, __uint_as_float(lw.x));
        }
    }
    // Clear the consumed words (own included) for the next call.
    for (int j = 0; j < nch; ++j) {
        const long long slot = slot0 + j;
        uint64_t *dst = p.ws_o + (slot * kHeadsPerCta + h) * HD;
#pragma unroll
        for (int k = 0; k < NP; ++k) st_part2(dst + sm.dim(k), 0ull, 0ull);
        if (sm.t == 0) st_part(p.ws_lse + slot * kHeadsPerCta + h, 0ull);
    }
    if (orow) {
        const float inv = 1.f / acc.s;
        float v[ND];
#pragma unroll
        for (int i = 0; i < ND; ++i) v[i] = acc.acc[i] * inv;
        put_out_pairs<NP, PEER>(p, orow + h * HD, sm.t, v);
    }
    return true;
}

template <int HD, bool FUSED, bool PEER = false, bool CLUSTER = false>
__global__ void __launch_bounds__(kThreads, HD == 64 ? 3 : 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const DecodeParams p) {
    static_assert(!(CLUSTER && PEER), "the cluster path serves one sequence on one GPU");
    using Cfg = DecodeCfg<HD>;
    constexpr int KSTEPS = HD / 16;

    __shared__ __align__(8) uint64_t full_bar[Cfg::kStages];
    __shared__ __align__(8) uint64_t empty_bar[Cfg::kStages];
    __shared__ __align__(8) uint64_t fin_bar;    // consumer-warp sync (bounded)
    __shared__ __align__(8) uint64_t epi_full;   // consumers -> epilogue: slots hold a chunk
    __shared__ __align__(8) uint64_t epi_empty;  // epilogue -> consumers: slots free again
    __shared__ __align__(8) uint64_t epi_exit;   // epilogue -> consumers: epilogue done
    __shared__ __align__(8) uint64_t merge_bar;  // consumers: partials copied into the ring
    __shared__ __align__(8) uint64_t q_full[2];  // fused: epilogue -> consumers, chunk inputs ready
    __shared__ StageMeta meta[Cfg::kStages];
    __shared__ EpiInfo epi;
    __shared__ long long s_total;
    __shared__ int s_b0;
    __shared__ long long s_pref_b0;
    __shared__ int s_abort;
    __shared__ int s_last;  // final chunk: this CTA arrived last on its segment
    // A non-final split chunk whose segment the epilogue warp found this CTA
    // last to finish: merged by the consumer threads after their final chunk.
    __shared__ struct { int valid, b, nh, head0, nch; long long slot0; } s_pend;
    // Cluster path: rank 0's gather barrier (every rank's slot, in bytes), and
    // whether rank 0 has seen all of them.
    __shared__ __align__(8) uint64_t cl_bar;
    __shared__ int s_cl_gathered;
    extern __shared__ uint8_t smem_raw[];

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int G = p.seg_per_seq;
    // Programmatic dependent launch (no-ops otherwise): let the next grid in the
    // stream be scheduled as our CTAs retire, and wait for the preceding grid
    // before touching its outputs.
    griddep_launch_dependents();
    if constexpr (CLUSTER) {
        // Every CTA's gather barrier exists before any CTA arrives on rank 0's.
        if (tid == 0) {
            // Rank 0 expects every rank's slot, in bytes (count 1: its own
            // arrival, which states them).
            mbar_init(&cl_bar, 1);
            if (cl_rank() == 0)
                mbar_arrive_expect_tx(&cl_bar, cl_size() * (uint32_t)(Cfg::kClSlotFloats * 4));
            s_cl_gathered = 0;
            fence_barrier_init();
        }
        cl_sync_all();
    }
    if (p.pdl_mode == 1) griddep_wait();
    const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem_gen = smem_raw + (smem_base - smem_u32(smem_raw));
    // Set-up scan scratch: the head of the stage ring, free until the first TMA.
    long long *s_part = reinterpret_cast<long long *>(smem_gen);
    // Fused: the q slots hold the epilogue's prepared chunk inputs instead,
    // double-buffered by chunk parity: q [2][8][HD], new K/V rows [2][2][HD].
    bf16 *q_prep = reinterpret_cast<bf16 *>(smem_gen + Cfg::kQOffset);
    bf16 *nk_rows = q_prep + 2 * kHeadsPerCta * HD;
    static_assert(Cfg::kStages * Cfg::kQBytes >= 2 * (kHeadsPerCta + 2) * HD * 2,
                  "prepared chunk inputs must fit the q slots");

    // ---- 1. total pages T and empty-sequence outputs ------------------------
    const int per = (p.batch + kThreads - 1) / kThreads;
    const int bs = min(p.batch, tid * per), be = min(p.batch, bs + per);
    long long mine = 0;
    // Do all sequences hold the same (non-zero) number of pages as sequence 0?
    const int pages0 = (seq_tokens(p, 0, false) + kBlockSize - 1) / kBlockSize;
    bool same = pages0 > 0;
    for (int b = bs; b < be; ++b) {
        const int pb = (seq_tokens(p, b, false) + kBlockSize - 1) / kBlockSize;
        mine += pb;
        same = same && pb == pages0;
    }
    s_part[tid] = mine;
    const bool uniform = __syncthreads_and(same) != 0;
    if (warp == 0) {  // exclusive scan of the kThreads partial sums
        constexpr int kPer = kThreads / 32;
        long long v[kPer], run = 0;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            v[k] = s_part[lane * kPer + k];
            run += v[k];
        }
        long long incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        long long ex = incl - run;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const long long x = v[k];
            s_part[lane * kPer + k] = ex;
            ex += x;
        }
        if (lane == 31) s_total = incl;
    }
    __syncthreads();
    const long long T = s_total * G;
    if (T == 0) {  // every sequence is empty: zero outputs, nothing else
        if (p.pdl_mode == 2) griddep_wait();
        zero_empty_outputs<HD, PEER>(p, blockIdx.x, gridDim.x, tid, kThreads);
        if constexpr (PEER) {
            fence_acq_rel_sys();
            __syncthreads();
            if (tid == 0) peer_arrive(p);
        }
        return;
    }
    int C = gridDim.x;
    {
        // Auto: at least kMinPagesPerCta pages per CTA, so that a short batch is
        // not split into more partials than its merge can absorb cheaply.
        const long long want = p.partition_tokens > 0
                                   ? (T * kBlockSize + p.partition_tokens - 1) / p.partition_tokens
                                   : (T + kMinPagesPerCta - 1) / kMinPagesPerCta;
        if (want < C) C = (int)(want < 1 ? 1 : want);
        if (T < C) C = (int)T;
        // Segments of equal length and several CTAs per segment (a short,
        // uniform batch such as one sequence): a multiple of the segment count
        // puts every range inside one segment, so that no CTA holds pieces of
        // two split segments (two merges in a row), at the cost of at most an
        // eighth of the CTAs.
        const long long S = uniform ? T / pages0 : 0;  // uniform: pages0 > 0
        if (uniform && p.partition_tokens == 0 && C >= 2 * S) {
            const long long Cs = S * (C / S);
            if ((C - Cs) * 8 <= C) C = (int)Cs;
        }
    }
    const int cta = blockIdx.x;
    long long start, end;
    if constexpr (CLUSTER) {
        // One sequence: cluster c takes segment c, its ranks one share each of
        // the segment's P pages. Rank r takes share (r + cs/2) mod cs, so that
        // the last share (the new token's page, and the extra page of an
        // uneven split) is not rank 0's, which also gathers. With P below the
        // cluster size rank r takes page r (rank 0 always holds one).
        C = gridDim.x;
        const long long cs = cl_size(), r = cl_rank(), P = pages0;
        const long long s0 = (long long)(cta / cs) * P;
        const long long c = P >= cs ? (r + cs / 2) % cs : r;
        start = s0 + (P >= cs ? c * P / cs : min(c, P));
        end = s0 + (P >= cs ? (c + 1) * P / cs : min(c + 1, P));
    } else {
        start = (long long)cta * T / C;
        end = (long long)(cta + 1) * T / C;
    }
    if (cta >= C || start >= end) {  // no pages: no outputs either
        if constexpr (PEER)
            if (tid == 0) peer_arrive(p);
        if constexpr (CLUSTER)
            if (tid < 128) cl_send_empty<HD>(tid, smem_u32(smem_gen + Cfg::kClOffset), &cl_bar);
        return;
    }
    // ---- 2. locate the sequence holding `start` -------------------------------
    {
        const long long lo = s_part[tid] * G;
        const long long hi = lo + mine * G;
        if (start >= lo && start < hi) {
            long long pref = lo;
            for (int b = bs; b < be; ++b) {
                const long long np =
                    (long long)((seq_tokens(p, b, false) + kBlockSize - 1) / kBlockSize) * G;
                if (start < pref + np) {
                    s_b0 = b;
                    s_pref_b0 = pref;
                    break;
                }
                pref += np;
            }
        }
    }
    // Order the scan's generic accesses to the ring before the TMA writes to it.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (tid == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kConsumerWarps);
        }
        mbar_init(&fin_bar, kConsumerWarps);
        mbar_init(&epi_full, 2);
        mbar_init(&epi_empty, 1);
        mbar_init(&epi_exit, 1);
        mbar_init(&merge_bar, 1);
        s_pend.valid = 0;
        mbar_init(&q_full[0], 1);
        mbar_init(&q_full[1], 1);
        s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        // ------------------------------------------------------ producer --
        if (p.pdl_mode == 2 && !FUSED) griddep_wait();
        if (lane == 0) {
            prefetch_tensormap(&tmap_k);
            prefetch_tensormap(&tmap_v);
        }
        ChunkCursor cur;
        cur.init(p, start, s_b0, s_pref_b0, lane == 0);
        Chunk ch;
        int it = 0;
        bool ok = true;
        while (ok && cur.next(p, end, lane == 0, ch)) {
            const int b = ch.b, g = ch.g, pg = ch.p0, take = ch.take;
            const bool final_chunk = cur.glob >= end;
            const int kvh = g / p.ctas_per_kv;
            const int hsub = g - kvh * p.ctas_per_kv;
            const int *trow = p.tables + (int64_t)b * p.table_stride;
            const int head0 = kvh * p.group + hsub * kHeadsPerCta;
            const int nh = min(kHeadsPerCta, p.group - hsub * kHeadsPerCta);
            for (int base = 0; base < take && ok; base += 32) {
                const int cnt = min(32, take - base);
                const int entry = lane < cnt ? __ldg(trow + pg + base + lane) : 0;
                for (int j = 0; j < cnt && ok; j += kPagesPerStage) {
                    const int np = min(kPagesPerStage, cnt - j);
                    int phys[kPagesPerStage];
#pragma unroll
                    for (int k = 0; k < kPagesPerStage; ++k)
                        phys[k] = __shfl_sync(0xffffffffu, entry, (j + k) & 31);
                    const int s = it % Cfg::kStages;
                    const bool first = base == 0 && j == 0;
                    if (lane == 0 && it >= Cfg::kStages &&
                        !mbar_wait_bounded(&empty_bar[s], ((it / Cfg::kStages) - 1) & 1, &s_abort,
                                           p.status))
                        ok = false;
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    uint32_t qbytes = 0;
                    if (lane == 0) {
                        if (!FUSED && first) {
                            qbytes = (uint32_t)(nh * HD * 2);
                            bulk_load(smem_gen + Cfg::kQOffset + s * Cfg::kQBytes,
                                      p.q + (int64_t)b * p.q_stride + (int64_t)head0 * HD, qbytes,
                                      &full_bar[s]);
                        }
                        uint8_t *kst = smem_gen + s * Cfg::kStageBytes;
                        for (int k = 0; k < np; ++k) {
                            int64_t row;
                            if (phys[k] < 0 || phys[k] >= p.num_blocks) {
                                set_status(p.status, LC_DEV_BAD_BLOCK);
                                row = p.pool_rows;  // wholly out of bounds: zero fill
                            } else {
                                row = page_row(phys[k], p.layer, kvh, p.num_layers, p.num_kv_heads);
                            }
                            uint8_t *kd = kst + k * Cfg::kPageBytes;
                            uint8_t *vd = kd + kPagesPerStage * Cfg::kPageBytes;
#pragma unroll
                            for (int h = 0; h < HD / 64; ++h) {
                                tma_load_2d(kd + h * 2048, &tmap_k, h * 64, (int)row, &full_bar[s]);
                                tma_load_2d(vd + h * 2048, &tmap_v, h * 64, (int)row, &full_bar[s]);
                            }
                        }
                    }
                    if (lane == 0) {
                        StageMeta &m = meta[s];
                        m.b = b;
                        m.g = g;
                        m.page0 = pg + base + j;
                        m.np = np;
                        m.n = ch.n;
                        m.pages_b = ch.pages_b;
                        const bool last_stage = base + j + np == take;
                        m.flags = (first ? kFirst : 0) | (last_stage ? kLast : 0) |
                                  (last_stage && final_chunk ? kFinal : 0);
                        m.chunk_p0 = pg;
                        m.take = take;
                        m.pos = FUSED ? __ldg(p.ctx_lens + b) + p.len_offset - 1 : -1;
                        m.seg_start = ch.seg_start;
                        // Copies may have landed already: the transaction count of a
                        // phase may run below zero until this arrival states it.
                        mbar_arrive_expect_tx(&full_bar[s],
                                              (uint32_t)(np * 2 * Cfg::kPageBytes) + qbytes);
                    }
                    ++it;
                }
            }
        }
        if (lane == 0 && ok) {  // end-of-range marker
            const int s = it % Cfg::kStages;
            if (it < Cfg::kStages || mbar_wait_bounded(&empty_bar[s], ((it / Cfg::kStages) - 1) & 1,
                                                       &s_abort, p.status)) {
                meta[s].flags = kDone;
                mbar_arrive(&full_bar[s]);
            }
        }
        if (lane == 0 && s_abort) {
            // A wait gave up: let the copies of the last stages land before exit.
            for (int k = it - Cfg::kStages; k < it; ++k)
                if (k >= 0) mbar_wait_drain(&full_bar[k % Cfg::kStages], (k / Cfg::kStages) & 1);
        }
        return;
    }

    float *red = reinterpret_cast<float *>(smem_gen + Cfg::kRedOffset);
    constexpr int kRedFloats = Cfg::kRedFloats;
    // Cluster path: two more warp-state slots past rank 0's gather buffer.
    float *red4 = reinterpret_cast<float *>(smem_gen + Cfg::kRed4Offset);

    if (warp == kEpilogueWarp) {
        // ------------------------------------------------------ epilogue --
        // Takes every chunk but the CTA's final one off the consumers' path:
        // combines the two half-CTA states, then writes the bf16 output (whole
        // segment) or, for a split segment (only the CTA's first chunk can be
        // one here), leaves its partial and counts it; if it came last, the
        // merge is left to the consumer threads (s_pend). The final chunk is
        // finished by the consumer threads themselves.
        constexpr int KD = HD / 32;  // head dims per lane
        // Fused: chunk j's inputs go to buffer j & 1. Before waiting for chunk k
        // to finish, chunks up to k + 1 are prepared; buffer (k + 1) & 1 was
        // last read by chunk k - 1, which has finished. The dependency wait
        // sits inside the first chunk's preparation.
        bool waited = !(FUSED && p.pdl_mode == 2);
        bool gated = !FUSED || p.gate == nullptr;
        if (p.pdl_mode == 2 && !FUSED) griddep_wait();
        ChunkCursor pcur;
        int prepared = 0;
        bool more = true;
        if constexpr (FUSED) pcur.init(p, start, s_b0, s_pref_b0, false);
        for (int k = 0;; ++k) {
            if constexpr (FUSED) {
                Chunk c;
                while (more && prepared <= k + 1) {
                    more = pcur.next(p, end, false, c);
                    if (!more) break;
                    const int qb = prepared & 1;
                    ChunkPrep<HD> cp;
                    cp.load_static(p, c, lane);
                    if (!waited) {
                        griddep_wait();
                        waited = true;
                    }
                    if (!gated) {
                        gate_wait(p.gate, &s_abort, p.status, lane);
                        gated = true;
                    }
                    cp.finish(p, c, q_prep + qb * kHeadsPerCta * HD, nk_rows + qb * 2 * HD,
                              &q_full[qb], lane);
                    ++prepared;
                }
                if (!waited) {
                    griddep_wait();
                    waited = true;
                }
            }
            if (k == 0) zero_empty_outputs<HD, PEER>(p, cta, C, lane, 32);
            if (!mbar_wait_bounded(&epi_full, k & 1, &s_abort, p.status)) break;
            const EpiInfo e = epi;
            if (e.done) break;
            float O[kHeadsPerCta][KD], Mh[kHeadsPerCta], Lh[kHeadsPerCta];
            const float *r0 = red, *r1 = red + kRedFloats;
#pragma unroll
            for (int h = 0; h < kHeadsPerCta; ++h) {
                const float m0 = r0[kHeadsPerCta * HD + h], m1 = r1[kHeadsPerCta * HD + h];
                const float l0 = r0[kHeadsPerCta * HD + kHeadsPerCta + h];
                const float l1 = r1[kHeadsPerCta * HD + kHeadsPerCta + h];
                const float M = fmaxf(m0, m1);
                const float u = M == -INFINITY ? 0.f : M;
                const float e0 = fast_exp2(m0 - u), e1 = fast_exp2(m1 - u);
                Mh[h] = M;
                Lh[h] = l0 * e0 + l1 * e1;
#pragma unroll
                for (int kk = 0; kk < KD; ++kk)
                    O[h][kk] = r0[h * HD + kk * 32 + lane] * e0 + r1[h * HD + kk * 32 + lane] * e1;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&epi_empty);  // the slots are free again
            if (e.whole) {
                bf16 *orow = p.out + (int64_t)e.b * p.out_stride + (int64_t)e.head0 * HD;
#pragma unroll
                for (int h = 0; h < kHeadsPerCta; ++h) {
                    if (h >= e.nh) break;
                    const float il = 1.f / Lh[h];
#pragma unroll
                    for (int kk = 0; kk < KD; ++kk)
                        put_out<PEER>(p, orow + h * HD + kk * 32 + lane,
                                      __float2bfloat16(O[h][kk] * il));
                }
                continue;
            }
            // Partial of a split segment in slot segment + this CTA, then its
            // arrival; the last piece to arrive merges.
            const long long slot = (long long)e.seg + cta;
            uint64_t *wo = p.ws_o + slot * kHeadsPerCta * HD;
#pragma unroll
            for (int h = 0; h < kHeadsPerCta; ++h) {
                const float il = 1.f / Lh[h];
#pragma unroll
                for (int kk = 0; kk < KD; ++kk) st_part(wo + h * HD + kk * 32 + lane, part_word(O[h][kk] * il));
                if (lane == h) st_part(p.ws_lse + slot * kHeadsPerCta + h, part_word(Mh[h] + __log2f(Lh[h])));
            }
            const int c_first = owner_cta(e.seg_start, T, C);
            const int nch = owner_cta(e.seg_start + e.pages_b - 1, T, C) - c_first + 1;
            int last = 0;
            if (lane == 0) last = atomicAdd(p.ws_cnt + e.seg, 1) == nch - 1;
            if (__shfl_sync(0xffffffffu, last, 0) && lane == 0) {
                p.ws_cnt[e.seg] = 0;  // ready for the next call
                s_pend.b = e.b;
                s_pend.nh = e.nh;
                s_pend.head0 = e.head0;
                s_pend.nch = nch;
                s_pend.slot0 = (long long)e.seg + c_first;
                s_pend.valid = 1;
            }
        }
        if constexpr (PEER) fence_acq_rel_sys();  // this warp's output stores
        __syncwarp();
        if (lane == 0) mbar_arrive(&epi_exit);
        return;
    }

    // ---------------------------------------------------------- consumers --
    const int g8 = lane >> 2, c4 = lane & 3;
    const int mi = lane >> 3, r8 = lane & 7;
    const int k_row = (mi & 1) * 8 + r8, k_chunk = mi >> 1;  // QK A operand (K tile)
    const int v_row = (mi >> 1) * 8 + r8, v_chunk = mi & 1;  // PV A operand (V^T tile)
    if (p.pdl_mode == 2) griddep_wait();
    uint32_t qf[KSTEPS][2];
    uint32_t fin_phase = 0, merge_phase = 0;
    bool cl_sent = false;  // cluster path: this thread's share is on its way to rank 0
    int chunk_idx = 0;  // chunks handed to the epilogue so far
    int nk_it = -1, nk_warp = -1;  // fused: stage and warp of the new token's page
    WarpState<HD> st;
    st.reset();
    for (int it = 0;; ++it) {
        const int s = it % Cfg::kStages;
        if (!mbar_wait_bounded(&full_bar[s], (it / Cfg::kStages) & 1, &s_abort, p.status)) break;
        const StageMeta m = meta[s];
        if (m.flags & kDone) {  // not reached: the final chunk ends the loop
            if (warp < 2) {  // tell the epilogue warp to finish
                if (chunk_idx > 0)
                    mbar_wait_bounded(&epi_empty, (chunk_idx - 1) & 1, &s_abort, p.status);
                if (warp == 0 && lane == 0) epi.done = 1;
                __syncwarp();
                if (lane == 0) mbar_arrive(&epi_full);
            }
            break;
        }
        const int kvh = m.g / p.ctas_per_kv;
        const int hsub = m.g - kvh * p.ctas_per_kv;
        const int nh = min(kHeadsPerCta, p.group - hsub * kHeadsPerCta);
        if (m.flags & kFirst) {
            const bool hv = g8 < nh;
            if constexpr (FUSED) {
                // q comes biased and rotated from the epilogue warp.
                const int qb = chunk_idx & 1;
                if (!mbar_wait_bounded(&q_full[qb], (chunk_idx >> 1) & 1, &s_abort, p.status)) break;
                const bf16 *qs = q_prep + qb * kHeadsPerCta * HD + g8 * HD + 2 * c4;
#pragma unroll
                for (int j = 0; j < KSTEPS; ++j) {
                    qf[j][0] = *reinterpret_cast<const uint32_t *>(qs + 16 * j);
                    qf[j][1] = *reinterpret_cast<const uint32_t *>(qs + 16 * j + 8);
                }
                // Does this chunk end with the new token's page, and which warp
                // and stage will hold it? Stages start at the chunk's first page.
                nk_it = -1;
                if (m.pos == m.n - 1 && m.chunk_p0 + m.take == m.pages_b) {
                    const int k = m.pages_b - 1 - m.chunk_p0;
                    nk_it = it + k / kPagesPerStage;
                    nk_warp = k % kPagesPerStage;
                }
            } else {
                const uint8_t *qs = smem_gen + Cfg::kQOffset + s * Cfg::kQBytes;
#pragma unroll
                for (int j = 0; j < KSTEPS; ++j) {
                    qf[j][0] = hv ? *reinterpret_cast<const uint32_t *>(qs + (g8 * HD + 16 * j + 2 * c4) * 2) : 0u;
                    qf[j][1] = hv ? *reinterpret_cast<const uint32_t *>(qs + (g8 * HD + 16 * j + 8 + 2 * c4) * 2) : 0u;
                }
            }
            st.reset();
        }
        if (warp < m.np) {
            const int page = m.page0 + warp;
            const int valid = min(kBlockSize, m.n - page * kBlockSize);
            const uint32_t kpage = smem_base + s * Cfg::kStageBytes + warp * Cfg::kPageBytes;
            const uint32_t vpage = kpage + kPagesPerStage * Cfg::kPageBytes;
            if (FUSED && it == nk_it && warp == nk_warp) {
                // The new token: its rotated K and V + bias (prepared by the
                // epilogue warp, which also appends them to the pools) replace
                // the tile row, which may have been loaded before the append.
                patch_new_row<HD>(nk_rows + (chunk_idx & 1) * 2 * HD, smem_gen, smem_base, kpage,
                                  vpage, m.pos % kBlockSize, lane);
                // Later bulk/TMA writes into this stage are async-proxy accesses.
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < KSTEPS; ++j) {
                uint32_t a[4];
                ldmatrix_x4(a, tile_addr(kpage, k_row, 2 * j + k_chunk));
                mma_bf16_16816(sc, a, qf[j][0], qf[j][1]);
            }
            // sc: (tok g8, head 2c4), (g8, 2c4+1), (g8+8, 2c4), (g8+8, 2c4+1)
            const float s0 = g8 < valid ? sc[0] * p.scale_log2 : -INFINITY;
            const float s1 = g8 < valid ? sc[1] * p.scale_log2 : -INFINITY;
            const float s2 = g8 + 8 < valid ? sc[2] * p.scale_log2 : -INFINITY;
            const float s3 = g8 + 8 < valid ? sc[3] * p.scale_log2 : -INFINITY;
            float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(st.m0, mx0), mn1 = fmaxf(st.m1, mx1);
            const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
            const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
            const float al0 = fast_exp2(st.m0 - mu0), al1 = fast_exp2(st.m1 - mu1);
            st.m0 = mn0;
            st.m1 = mn1;
            const float p0 = fast_exp2(s0 - mu0), p1 = fast_exp2(s1 - mu1);
            const float p2 = fast_exp2(s2 - mu0), p3 = fast_exp2(s3 - mu1);
            st.l0 = st.l0 * al0 + (p0 + p2);
            st.l1 = st.l1 * al1 + (p1 + p3);
#pragma unroll
            for (int i = 0; i < KSTEPS; ++i) {
                st.o[i][0] *= al0;
                st.o[i][1] *= al1;
                st.o[i][2] *= al0;
                st.o[i][3] *= al1;
            }
            const uint32_t b0 = movmatrix_trans(pack_bf16(p0, p1));
            const uint32_t b1 = movmatrix_trans(pack_bf16(p2, p3));
#pragma unroll
            for (int i = 0; i < KSTEPS; ++i) {
                uint32_t a[4];
                ldmatrix_x4_trans(a, tile_addr(vpage, v_row, 2 * i + v_chunk));
                mma_bf16_16816(st.o[i], a, b0, b1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        if (!(m.flags & kLast)) continue;

        // ---------------------------------------------- finish the chunk --
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {  // l over the 8 token lanes of a head
            st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, off);
            st.l1 += __shfl_xor_sync(0xffffffffu, st.l1, off);
        }
        // Halve the 4 warp states into the 2 shared slots. Every chunk but the
        // CTA's final one is then handed to the epilogue warp; for the final
        // one the epilogue is only told to finish.
        const bool final_chunk = (m.flags & kFinal) != 0;
        // Cluster path: a CTA holds one chunk, its final one. The four warp
        // states go to four slots at once (no halving round), and the
        // epilogue warp is only told to finish.
        const bool four = CLUSTER && final_chunk;
        if (chunk_idx > 0) mbar_wait_bounded(&epi_empty, (chunk_idx - 1) & 1, &s_abort, p.status);
        if (four) {
            state_store<HD>(warp < 2 ? red + warp * kRedFloats
                                     : red4 + (warp - 2) * kRedFloats, st, lane);
            if (warp < 2) {  // epi_full counts warps 0 and 1
                if (warp == 0 && lane == 0) epi.done = 1;
                __syncwarp();
                if (lane == 0) mbar_arrive(&epi_full);
            }
        } else if (warp >= 2) {
            state_store<HD>(red + (warp - 2) * kRedFloats, st, lane);
        }
        if (!four) consumer_sync(&fin_bar, fin_phase, &s_abort, p.status);
        if (!four && warp < 2) {
            state_combine<HD>(st, red + warp * kRedFloats, lane);
            __syncwarp();
            state_store<HD>(red + warp * kRedFloats, st, lane);
            if (warp == 0 && lane == 0) {
                epi.b = m.b;
                epi.seg = m.b * G + m.g;
                epi.nh = nh;
                epi.head0 = kvh * p.group + hsub * kHeadsPerCta;
                epi.pages_b = m.pages_b;
                epi.whole = m.chunk_p0 == 0 && m.take == m.pages_b;
                epi.done = final_chunk;
                epi.seg_start = m.seg_start;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&epi_full);
        }
        ++chunk_idx;
        st.reset();
        if (!final_chunk) continue;

        // ------------------------------------- the final chunk, 128 threads --
        // Thread ct owns head ct >> 4 and dim pairs 32k + 2 (ct & 15) of the
        // CTA's state for this chunk: whole segment -> output; split segment ->
        // partial + arrival, and the merge if this CTA came last.
        consumer_sync(&fin_bar, fin_phase, &s_abort, p.status);  // both (four) slots stored
        constexpr int NP = ShareMap<HD>::NP, ND = ShareMap<HD>::ND;
        const ShareMap<HD> sm(warp * 32 + lane);
        // Slots in order: red[0], red[1] (and red4[0], red4[1] in the cluster path).
        constexpr int NS = CLUSTER ? 4 : 2;
        const float *rs[NS];
        rs[0] = red;
        rs[1] = red + kRedFloats;
        if constexpr (CLUSTER) {
            rs[2] = red4;
            rs[3] = red4 + kRedFloats;
        }
        float mj[NS], ej[NS];
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < NS; ++j) {
            mj[j] = rs[j][kHeadsPerCta * HD + sm.h];
            M = fmaxf(M, mj[j]);
        }
        const float u = M == -INFINITY ? 0.f : M;
        float Ls = 0.f;
#pragma unroll
        for (int j = 0; j < NS; ++j) {
            ej[j] = fast_exp2(mj[j] - u);
            Ls += rs[j][kHeadsPerCta * HD + kHeadsPerCta + sm.h] * ej[j];
        }
        const float il = 1.f / Ls;
        float o[ND];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            float x = 0.f, y = 0.f;
#pragma unroll
            for (int j = 0; j < NS; ++j) {
                const float2 a = *reinterpret_cast<const float2 *>(rs[j] + sm.h * HD + sm.dim(k));
                x += a.x * ej[j];
                y += a.y * ej[j];
            }
            o[2 * k] = x * il;
            o[2 * k + 1] = y * il;
        }
        bf16 *orow = sm.h < nh ? p.out + (int64_t)m.b * p.out_stride +
                                     (int64_t)(kvh * p.group + hsub * kHeadsPerCta) * HD
                               : nullptr;
        if constexpr (CLUSTER) {
            // The piece goes to slot `rank` of rank 0's gather buffer; rank 0
            // combines the slots in rank order once every rank's bytes have
            // landed.
            const uint32_t rank = cl_rank();
            cl_send<HD>(warp * 32 + lane, o, M + __log2f(Ls), smem_u32(smem_gen + Cfg::kClOffset),
                        &cl_bar);
            cl_sent = true;
            if (rank == 0) {
                mbar_wait_drain(&cl_bar, 0);  // bounded by time alone
                const bool all = mbar_try_wait(&cl_bar, 0);
                if (warp == 0 && lane == 0) s_cl_gathered = all;
                if (all && orow) {
                    // Two passes over the slots, every load of a pass in flight at
                    // once: the largest log2-sum-exp, then the weighted sum in rank
                    // order (slots with -inf, CTAs without pages, weigh nothing).
                    const float *bl = reinterpret_cast<const float *>(smem_gen + Cfg::kClOffset);
                    const int cs = (int)cl_size();
                    float lj[kClusterMax];
                    float mx = -INFINITY;
#pragma unroll
                    for (int j = 0; j < kClusterMax; ++j) {
                        lj[j] = j < cs ? bl[j * Cfg::kClSlotFloats + kHeadsPerCta * HD + sm.h] : -INFINITY;
                        mx = fmaxf(mx, lj[j]);
                    }
                    float ssum = 0.f, acc[ND];
#pragma unroll
                    for (int i = 0; i < ND; ++i) acc[i] = 0.f;
#pragma unroll
                    for (int j = 0; j < kClusterMax; ++j) {
                        if (lj[j] == -INFINITY) continue;
                        const float w = fast_exp2(lj[j] - mx);
                        ssum += w;
                        const float *sl = bl + j * Cfg::kClSlotFloats + sm.h * HD;
#pragma unroll
                        for (int k = 0; k < NP; ++k) {
                            const float2 x = *reinterpret_cast<const float2 *>(sl + sm.dim(k));
                            acc[2 * k] = fmaf(w, x.x, acc[2 * k]);
                            acc[2 * k + 1] = fmaf(w, x.y, acc[2 * k + 1]);
                        }
                    }
                    const float inv = 1.f / ssum;
#pragma unroll
                    for (int i = 0; i < ND; ++i) acc[i] *= inv;
                    put_out_pairs<NP, PEER>(p, orow + sm.h * HD, sm.t, acc);
                }
            }
            break;
        }
        if (m.chunk_p0 == 0 && m.take == m.pages_b) {
            if (orow) put_out_pairs<NP, PEER>(p, orow + sm.h * HD, sm.t, o);
            break;
        }
        const int seg = m.b * G + m.g;
        const long long slot = (long long)seg + cta;
        const float lse = M + __log2f(Ls);
        {
            uint64_t *wo = p.ws_o + (slot * kHeadsPerCta + sm.h) * HD;
#pragma unroll
            for (int k = 0; k < NP; ++k)
                st_part2(wo + sm.dim(k), part_word(o[2 * k]), part_word(o[2 * k + 1]));
            if (sm.t == 0) st_part(p.ws_lse + slot * kHeadsPerCta + sm.h, part_word(lse));
        }
        const int c_first = owner_cta(m.seg_start, T, C);
        const int nch = owner_cta(m.seg_start + m.pages_b - 1, T, C) - c_first + 1;
        if (warp == 0 && lane == 0) s_last = atomicAdd(p.ws_cnt + seg, 1) == nch - 1;
        consumer_sync(&fin_bar, fin_phase, &s_abort, p.status);
        if (s_last && !s_abort) {
            if (warp == 0 && lane == 0) p.ws_cnt[seg] = 0;  // ready for the next call
            merge_split_segment<HD, PEER>(p, (long long)seg + c_first, nch, cta - c_first, o, lse,
                                          sm, orow, smem_gen, &merge_bar, merge_phase,
                                          &fin_bar, fin_phase, &s_abort, warp == 0 && lane == 0);
        }
        break;
    }

    // ---------------------------------------------------------------- exit --
    // A segment the epilogue warp found this CTA last to finish (its first
    // chunk) is merged here, once the epilogue is done.
    mbar_wait_bounded(&epi_exit, 0, &s_abort, p.status);
    if (s_pend.valid && !s_abort &&
        consumer_sync(&fin_bar, fin_phase, &s_abort, p.status)) {  // the ring is free again
        const ShareMap<HD> sm(warp * 32 + lane);
        float none[HD / 16] = {};
        bf16 *orow = sm.h < s_pend.nh
                         ? p.out + (int64_t)s_pend.b * p.out_stride + (int64_t)s_pend.head0 * HD
                         : nullptr;
        merge_split_segment<HD, PEER>(p, s_pend.slot0, s_pend.nch, -1, none, 0.f, sm, orow,
                                      smem_gen, &merge_bar, merge_phase, &fin_bar,
                                      fin_phase, &s_abort, warp == 0 && lane == 0);
    }
    if constexpr (PEER) {
        fence_acq_rel_sys();  // this thread's output stores, then one arrival per CTA
        consumer_sync(&fin_bar, fin_phase, &s_abort, p.status);
        if (warp == 0 && lane == 0) peer_arrive(p);
    }
    if constexpr (CLUSTER) {
        // Every consumer thread sends its share of the slot exactly once (an
        // empty share if its piece was not sent), and rank 0 stays until all
        // bytes have landed: they land in its shared memory.
        if (!cl_sent) cl_send_empty<HD>(warp * 32 + lane, smem_u32(smem_gen + Cfg::kClOffset), &cl_bar);
        if (warp == 0 && lane == 0 && cl_rank() == 0 && !s_cl_gathered) mbar_wait_drain(&cl_bar, 0);
    }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace layout: counters [batch*segments] int32 | lse [slots][8] and
// o [slots][8][hd] as tagged 64-bit words (value, tag), with slots = persistent
// CTAs + batch*segments (slot of a piece = its segment + its CTA).
struct WsLayout {
    size_t cnt_bytes, lse_bytes, o_bytes;
    size_t total() const { return cnt_bytes + lse_bytes + o_bytes; }
};

WsLayout ws_layout(int batch, int segments_per_seq, int hd, int max_ctas) {
    const size_t segs = (size_t)batch * segments_per_seq;
    const size_t slots = segs + (size_t)max_ctas;
    WsLayout l;
    l.cnt_bytes = align256(segs * 4);
    l.lse_bytes = align256(slots * kHeadsPerCta * 8);
    l.o_bytes = slots * kHeadsPerCta * hd * 8;
    return l;
}

int segments_per_seq(int hq, int hkv) {
    const int group = hq / hkv;
    return hkv * ((group + kHeadsPerCta - 1) / kHeadsPerCta);
}

// Persistent grid: resident CTAs per SM for this head_dim, times the SM count.
// Without a usable device (host-only callers sizing a workspace) a B200's
// 148 SMs are assumed.
template <int HD>
int max_ctas_for_device() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = -1;
    }
    const int idx = dev < 0 || dev >= 64 ? 0 : dev;
    if (!cached[idx] || dev < 0) {
        int per_sm = 0;
        const int smem = DecodeCfg<HD>::kSmemBytes;
        if (dev < 0 ||
            ensure_smem_attr((const void *)paged_decode_kernel<HD, false>, smem) != LC_OK ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_kernel<HD, false>,
                                                          kThreads, smem) != cudaSuccess ||
            per_sm < 1) {
            cudaGetLastError();
            per_sm = HD == 64 ? 3 : 2;
        }
        const int n = per_sm * sm_count();
        if (dev < 0) return n;
        cached[idx] = n;
    }
    return cached[idx];
}

int max_ctas(int hd) { return hd == 64 ? max_ctas_for_device<64>() : max_ctas_for_device<128>(); }

template <int HD, bool FUSED = false, bool PEER = false>
int launch_decode(const DecodeParams &prm, int grid, const void *k_pool, const void *v_pool,
                  cudaStream_t stream) {
    CUtensorMap mk, mv;
    int rc = pool_tensor_map(k_pool, prm.pool_rows, HD, &mk);
    if (rc) return rc;
    rc = pool_tensor_map(v_pool, prm.pool_rows, HD, &mv);
    if (rc) return rc;
    const int smem = DecodeCfg<HD>::kSmemBytes;
    rc = ensure_smem_attr((const void *)paged_decode_kernel<HD, FUSED, PEER>, smem);
    if (rc) return rc;
    const int mode = dependent_launch_mode();
    DecodeParams prm2 = prm;
    prm2.pdl_mode = mode;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = mode > 0 ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, paged_decode_kernel<HD, FUSED, PEER>, mk, mv, prm2) !=
        cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    return LC_OK;
}

// Single-sequence decode (fused or not) over clusters of `cs` CTAs, one
// cluster per segment (grid = segments x cs). Returns LC_ERR_NOT_SUPPORTED,
// launching nothing, when the device cannot run such clusters.
template <int HD, bool FUSED>
int launch_decode_cluster(const DecodeParams &prm, int segments, int cs, const void *k_pool,
                          const void *v_pool, cudaStream_t stream) {
    auto kern = paged_decode_kernel<HD, FUSED, false, true>;
    const int smem = DecodeCfg<HD>::kSmemClusterBytes;
    CUtensorMap mk, mv;
    int rc = pool_tensor_map(k_pool, prm.pool_rows, HD, &mk);
    if (rc) return rc;
    rc = pool_tensor_map(v_pool, prm.pool_rows, HD, &mv);
    if (rc) return rc;
    static std::mutex mu;
    static int fits[64][kClusterMax + 1];  // 0 unknown, 1 yes, -1 no; per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LC_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(segments * cs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (fits[dev][cs] == 0) {
            int n = 0;
            cfg.numAttrs = 1;
            const bool ok =
                ensure_smem_attr((const void *)kern, smem) == LC_OK &&
                (cs <= 8 || cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed,
                                                 1) == cudaSuccess) &&
                cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n >= 1;
            cudaGetLastError();
            fits[dev][cs] = ok ? 1 : -1;
        }
        if (fits[dev][cs] < 0) return LC_ERR_NOT_SUPPORTED;
    }
    const int mode = dependent_launch_mode();
    DecodeParams prm2 = prm;
    prm2.pdl_mode = mode;
    cfg.numAttrs = mode > 0 ? 2 : 1;
    if (cudaLaunchKernelEx(&cfg, kern, mk, mv, prm2) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    return LC_OK;
}

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" size_t lc_paged_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                                 int head_dim) {
    if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads)
        return 0;
    if (head_dim != 64 && head_dim != 128) return 0;
    return ws_layout(batch, segments_per_seq(num_q_heads, num_kv_heads), head_dim,
                     max_ctas(head_dim))
        .total();
}

extern "C" int lc_paged_decode_workspace_init(void *workspace, size_t workspace_bytes,
                                              lc_stream_t stream) {
    if (!workspace && workspace_bytes) return LC_ERR_INVALID_ARGUMENT;
    if (!workspace_bytes) return LC_OK;
    return cudaMemsetAsync(workspace, 0, workspace_bytes, as_stream(stream)) == cudaSuccess
               ? LC_OK
               : LC_ERR_CUDA;
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
        len_offset > 1 || partition_tokens < 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if (batch == 0) return LC_OK;
    if (!aligned16(k_pool) || !aligned16(v_pool) || !aligned16(q) || (q_stride & 7) ||
        ((uintptr_t)out & 1))
        return LC_ERR_MISALIGNED;
    if (q_stride < (int64_t)num_q_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim)
        return LC_ERR_INVALID_ARGUMENT;
    const int64_t pool_rows = num_blocks * num_layers * num_kv_heads * kBlockSize;
    if (pool_rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;

    const int G = segments_per_seq(num_q_heads, num_kv_heads);
    const int cmax = max_ctas(head_dim);
    const WsLayout wl = ws_layout(batch, G, head_dim, cmax);
    if (!workspace || workspace_bytes < wl.total()) return LC_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned16(workspace)) return LC_ERR_MISALIGNED;
    // Grid: the persistent size, trimmed when the host's context hint shows
    // there is less work than two pages per CTA.
    int grid = cmax;
    if (max_context_len > 0) {
        const long long pages_hint =
            (long long)batch * G * ((max_context_len + kBlockSize - 1) / kBlockSize);
        const long long want = (pages_hint + kMinPagesPerCta - 1) / kMinPagesPerCta;
        if (want < grid) grid = (int)(want < 1 ? 1 : want);
    }
    DecodeParams prm{};
    prm.out = (bf16 *)out;
    prm.out_stride = out_stride;
    prm.q = (const bf16 *)q;
    prm.q_stride = q_stride;
    prm.tables = block_tables;
    prm.table_stride = table_stride;
    prm.ctx_lens = context_lens;
    prm.len_offset = len_offset;
    prm.batch = batch;
    prm.pool_rows = pool_rows;
    prm.num_blocks = num_blocks;
    prm.num_layers = num_layers;
    prm.layer = layer;
    prm.num_q_heads = num_q_heads;
    prm.num_kv_heads = num_kv_heads;
    prm.group = num_q_heads / num_kv_heads;
    prm.ctas_per_kv = (prm.group + kHeadsPerCta - 1) / kHeadsPerCta;
    prm.seg_per_seq = G;
    prm.partition_tokens = partition_tokens;
    prm.scale_log2 = sm_scale * 1.4426950408889634f;
    uint8_t *ws = (uint8_t *)workspace;
    prm.ws_cnt = (int *)ws;
    prm.ws_lse = (uint64_t *)(ws + wl.cnt_bytes);
    prm.ws_o = (uint64_t *)(ws + wl.cnt_bytes + wl.lse_bytes);
    prm.status = dev_status;
    prm.out_vec = ((uintptr_t)out & 3) == 0 && out_stride % 2 == 0;
    cudaStream_t s = as_stream(stream);
    // One sequence (lc_flash_decoding, the reference-shaped entry, always):
    // each segment's pages over one thread-block cluster, as in
    // lc_rope_append_decode.
    if (batch == 1 && partition_tokens == 0 && max_context_len > 0) {
        const int pages = (max_context_len + kBlockSize - 1) / kBlockSize;
        const int cs = min(kClusterMax, pages / kClusterMinPages);
        if (cs >= 2) {
            const int rc = head_dim == 64
                               ? launch_decode_cluster<64, false>(prm, G, cs, k_pool, v_pool, s)
                               : launch_decode_cluster<128, false>(prm, G, cs, k_pool, v_pool, s);
            if (rc != LC_ERR_NOT_SUPPORTED) return rc;
        }
    }
    return head_dim == 64 ? launch_decode<64>(prm, grid, k_pool, v_pool, s)
                          : launch_decode<128>(prm, grid, k_pool, v_pool, s);
}

static int rope_append_decode_impl(void *out, int64_t out_stride, const void *qkv,
                                   int64_t row_stride, const int *positions,
                                   const void *q_bias, const void *k_bias, const void *v_bias,
                                   const float *cos_cache, const float *sin_cache,
                                   int rope_rows, void *k_pool, void *v_pool,
                                   int64_t num_blocks, int num_layers, int layer,
                                   int num_q_heads, int num_kv_heads, int head_dim,
                                   const int *block_tables, int table_stride, int batch,
                                   int max_context_len, int partition_tokens, float sm_scale,
                                   void *workspace, size_t workspace_bytes, int *dev_status,
                                   lc_stream_t stream, const int *gate,
                                   const lc_peer_group *group);

extern "C" int lc_rope_append_decode(void *out, int64_t out_stride, const void *qkv,
                                     int64_t row_stride, const int *positions,
                                     const void *q_bias, const void *k_bias, const void *v_bias,
                                     const float *cos_cache, const float *sin_cache,
                                     int rope_rows, void *k_pool, void *v_pool,
                                     int64_t num_blocks, int num_layers, int layer,
                                     int num_q_heads, int num_kv_heads, int head_dim,
                                     const int *block_tables, int table_stride, int batch,
                                     int max_context_len, int partition_tokens, float sm_scale,
                                     void *workspace, size_t workspace_bytes, int *dev_status,
                                     lc_stream_t stream) {
    return rope_append_decode_impl(out, out_stride, qkv, row_stride, positions, q_bias, k_bias,
                                   v_bias, cos_cache, sin_cache, rope_rows, k_pool, v_pool,
                                   num_blocks, num_layers, layer, num_q_heads, num_kv_heads,
                                   head_dim, block_tables, table_stride, batch, max_context_len,
                                   partition_tokens, sm_scale, workspace, workspace_bytes,
                                   dev_status, stream, nullptr, nullptr);
}

extern "C" int lc_rope_append_decode_gated(
    void *out, int64_t out_stride, const void *qkv, int64_t row_stride, const int *positions,
    const void *q_bias, const void *k_bias, const void *v_bias, const float *cos_cache,
    const float *sin_cache, int rope_rows, void *k_pool, void *v_pool, int64_t num_blocks,
    int num_layers, int layer, int num_q_heads, int num_kv_heads, int head_dim,
    const int *block_tables, int table_stride, int batch, int max_context_len,
    int partition_tokens, float sm_scale, void *workspace, size_t workspace_bytes,
    int *dev_status, const int *gate, lc_stream_t stream) {
    if (!gate) return LC_ERR_INVALID_ARGUMENT;
    return rope_append_decode_impl(out, out_stride, qkv, row_stride, positions, q_bias, k_bias,
                                   v_bias, cos_cache, sin_cache, rope_rows, k_pool, v_pool,
                                   num_blocks, num_layers, layer, num_q_heads, num_kv_heads,
                                   head_dim, block_tables, table_stride, batch, max_context_len,
                                   partition_tokens, sm_scale, workspace, workspace_bytes,
                                   dev_status, stream, gate, nullptr);
}

extern "C" int lc_rope_append_decode_peer(
    void *out, int64_t out_stride, const void *qkv, int64_t row_stride, const int *positions,
    const void *q_bias, const void *k_bias, const void *v_bias, const float *cos_cache,
    const float *sin_cache, int rope_rows, void *k_pool, void *v_pool, int64_t num_blocks,
    int num_layers, int layer, int num_q_heads, int num_kv_heads, int head_dim,
    const int *block_tables, int table_stride, int batch, int max_context_len,
    int partition_tokens, float sm_scale, void *workspace, size_t workspace_bytes,
    int *dev_status, const lc_peer_group *group, lc_stream_t stream) {
    if (!group) return LC_ERR_INVALID_ARGUMENT;
    return rope_append_decode_impl(out, out_stride, qkv, row_stride, positions, q_bias, k_bias,
                                   v_bias, cos_cache, sin_cache, rope_rows, k_pool, v_pool,
                                   num_blocks, num_layers, layer, num_q_heads, num_kv_heads,
                                   head_dim, block_tables, table_stride, batch, max_context_len,
                                   partition_tokens, sm_scale, workspace, workspace_bytes,
                                   dev_status, stream, nullptr, group);
}

static int rope_append_decode_impl(void *out, int64_t out_stride, const void *qkv,
                                     int64_t row_stride, const int *positions,
                                     const void *q_bias, const void *k_bias, const void *v_bias,
                                     const float *cos_cache, const float *sin_cache,
                                     int rope_rows, void *k_pool, void *v_pool,
                                     int64_t num_blocks, int num_layers, int layer,
                                     int num_q_heads, int num_kv_heads, int head_dim,
                                     const int *block_tables, int table_stride, int batch,
                                     int max_context_len, int partition_tokens, float sm_scale,
                                     void *workspace, size_t workspace_bytes, int *dev_status,
                                     lc_stream_t stream, const int *gate,
                                     const lc_peer_group *group) {
    if (!out || !qkv || !positions || !q_bias || !k_bias || !v_bias || !cos_cache ||
        !sin_cache || !k_pool || !v_pool || !block_tables)
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (batch < 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || num_q_heads <= 0 ||
        num_kv_heads <= 0 || num_blocks <= 0 || table_stride <= 0 || rope_rows <= 0 ||
        partition_tokens < 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if (batch == 0 && !group) return LC_OK;  // a peer launch still signals its peers
    if (!aligned16(k_pool) || !aligned16(v_pool) || !aligned16(qkv) || (row_stride & 7) ||
        ((uintptr_t)out & 1))
        return LC_ERR_MISALIGNED;
    if (row_stride < (int64_t)(num_q_heads + 2 * num_kv_heads) * head_dim ||
        out_stride < (int64_t)num_q_heads * head_dim)
        return LC_ERR_INVALID_ARGUMENT;
    const int64_t pool_rows = num_blocks * num_layers * num_kv_heads * kBlockSize;
    if (pool_rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;

    const int G = segments_per_seq(num_q_heads, num_kv_heads);
    const int cmax = max_ctas(head_dim);
    const WsLayout wl = ws_layout(batch, G, head_dim, cmax);
    if (!workspace || workspace_bytes < wl.total()) return LC_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned16(workspace)) return LC_ERR_MISALIGNED;
    int grid = cmax;
    if (max_context_len > 0) {
        const long long pages_hint =
            (long long)batch * G * ((max_context_len + kBlockSize - 1) / kBlockSize);
        const long long want = (pages_hint + kMinPagesPerCta - 1) / kMinPagesPerCta;
        if (want < grid) grid = (int)(want < 1 ? 1 : want);
    }
    DecodeParams prm{};
    prm.out = (bf16 *)out;
    prm.out_stride = out_stride;
    prm.q = (const bf16 *)qkv;
    prm.q_stride = row_stride;
    prm.tables = block_tables;
    prm.table_stride = table_stride;
    prm.ctx_lens = positions;
    prm.len_offset = 1;
    prm.batch = batch;
    prm.pool_rows = pool_rows;
    prm.num_blocks = num_blocks;
    prm.num_layers = num_layers;
    prm.layer = layer;
    prm.num_q_heads = num_q_heads;
    prm.num_kv_heads = num_kv_heads;
    prm.group = num_q_heads / num_kv_heads;
    prm.ctas_per_kv = (prm.group + kHeadsPerCta - 1) / kHeadsPerCta;
    prm.seg_per_seq = G;
    prm.partition_tokens = partition_tokens;
    prm.scale_log2 = sm_scale * 1.4426950408889634f;
    uint8_t *ws = (uint8_t *)workspace;
    prm.ws_cnt = (int *)ws;
    prm.ws_lse = (uint64_t *)(ws + wl.cnt_bytes);
    prm.ws_o = (uint64_t *)(ws + wl.cnt_bytes + wl.lse_bytes);
    prm.status = dev_status;
    prm.out_vec = ((uintptr_t)out & 3) == 0 && out_stride % 2 == 0;
    prm.qkv = (const bf16 *)qkv;
    prm.q_bias = (const bf16 *)q_bias;
    prm.k_bias = (const bf16 *)k_bias;
    prm.v_bias = (const bf16 *)v_bias;
    prm.cos_t = cos_cache;
    prm.sin_t = sin_cache;
    prm.rope_rows = rope_rows;
    prm.k_pool_w = (bf16 *)k_pool;
    prm.v_pool_w = (bf16 *)v_pool;
    prm.gate = gate;
    cudaStream_t s = as_stream(stream);
    if (group) {
        // out's rows must lie in this rank's region past the signal words; the
        // same offsets address them in every peer's region.
        const uint8_t *base = group->region[group->rank];
        const uint8_t *lo = (const uint8_t *)out;
        const int64_t rows = batch > 0 ? batch : 1;
        const uint8_t *hi =
            lo + ((rows - 1) * out_stride + (int64_t)num_q_heads * head_dim) * 2;
        if (lo < base + LC_PEER_SIGNAL_BYTES || hi > base + group->bytes)
            return LC_ERR_INVALID_ARGUMENT;
        int *words = (int *)group->region[group->rank];
        prm.peer_done = words + kPeerDoneWord;
        prm.peer_seq = words + kPeerSeqWord;
        for (int r = 0; r < group->world; ++r) {
            if (r == group->rank) continue;
            prm.peer_delta[prm.n_peer] = (long long)(group->region[r] - base);
            prm.peer_flag[prm.n_peer] = (int *)group->region[r] + group->rank;
            ++prm.n_peer;
        }
        return head_dim == 64 ? launch_decode<64, true, true>(prm, grid, k_pool, v_pool, s)
                              : launch_decode<128, true, true>(prm, grid, k_pool, v_pool, s);
    }
    // One sequence: each segment's pages over a cluster of up to kClusterMax
    // CTAs (at least 4 pages each), merged in rank 0's shared memory instead
    // of through the workspace.
    if (batch == 1 && partition_tokens == 0 && max_context_len > 0) {
        const int pages = (max_context_len + kBlockSize - 1) / kBlockSize;
        const int cs = min(kClusterMax, pages / kClusterMinPages);
        if (cs >= 2) {
            const int rc = head_dim == 64
                               ? launch_decode_cluster<64, true>(prm, G, cs, k_pool, v_pool, s)
                               : launch_decode_cluster<128, true>(prm, G, cs, k_pool, v_pool, s);
            if (rc != LC_ERR_NOT_SUPPORTED) return rc;
        }
    }
    return head_dim == 64 ? launch_decode<64, true>(prm, grid, k_pool, v_pool, s)
                          : launch_decode<128, true>(prm, grid, k_pool, v_pool, s);
}

extern "C" size_t lc_flash_decoding_workspace_size(int num_q_heads, int head_dim,
                                                   int max_seq_len) {
    (void)max_seq_len;  // the persistent split needs no per-length storage
    // Hq bounds the number of (kv head, 8-head slice) segments of one sequence.
    if (num_q_heads <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
    return ws_layout(1, num_q_heads, head_dim, max_ctas(head_dim)).total();
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
    if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads)
        return num_q_heads > 0 && num_kv_heads > 0 ? LC_ERR_UNSUPPORTED_SHAPE
                                                   : LC_ERR_INVALID_ARGUMENT;
    // The reference's table holds ceil(max_position_embeddings / 16) entries
    // (src/layers/kv_cache.rs:70-71).
    int table_len = (max_seq_len + kBlockSize - 1) / kBlockSize;
    if (table_len < host_pos / kBlockSize + 1) table_len = host_pos / kBlockSize + 1;
    const int64_t stride = (int64_t)num_q_heads * head_dim;
    // The workspace was sized with Hq segments; the call needs Hkv*ceil(group/8).
    return lc_paged_decode(output, stride, q, stride, k_pool, v_pool, num_physical_blocks,
                           num_layers, layer_idx, num_q_heads, num_kv_heads, head_dim,
                           block_table, table_len, current_pos, /*len_offset=*/1, 1,
                           host_pos + 1, 0, sm_scale, workspace, workspace_bytes, nullptr,
                           stream);
}

// ---------------------------------------------------------------------------
// Allocation-free entry point: lc_paged_decode_static.
//
// lc_paged_decode needs a caller-allocated workspace. Some callers cannot
// allocate device memory when they decode: a serving loop that must never hit
// cudaMalloc/cudaFree (they can synchronise the whole device and stall every
// other stream mid-step), a host engine whose device memory is entirely
// reserved up front for its own KV pools and buffers, or an embedding runtime
// that only hands the attention plugin raw tensor pointers and a stream. For
// them the split-K scratch lives in the fixed device array below, which every
// GPU that loads this library holds (LC_PAGED_DECODE_STATIC_SCRATCH_BYTES) until
// the process exits.
//
// Host code cannot use the array's name as a device address (it names a host
// shadow); the first call on each device resolves the real address with
// cudaGetSymbolAddress while that device is current and caches it. Calls share
// the array and it keeps the last call's contents: each call clears the part
// it uses (arrival counters and tagged partials) before its launch, and calls
// that overlap on the same GPU (issued on two streams, say) race on it. Each
// device has its own copy of the array.
static __device__ __align__(256) unsigned char
    lc_static_decode_scratch[LC_PAGED_DECODE_STATIC_SCRATCH_BYTES];

namespace lc {
namespace {

constexpr int kStaticMaxDevices = 64;

struct StaticDecodeSetup {
    void *scratch;
    int max_ctas64, max_ctas128;
    bool ready;
};
StaticDecodeSetup g_static_setup[kStaticMaxDevices];
std::mutex g_static_mu;

template <int HD>
int static_max_ctas(int sms, int *out) {
    const int smem = DecodeCfg<HD>::kSmemBytes;
    int per_sm = 0;
    if (cudaFuncSetAttribute(paged_decode_kernel<HD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_kernel<HD, false>, kThreads,
                                                      smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    *out = per_sm * sms;
    return LC_OK;
}

// One-time set-up of the current device `dev` (must be current).
int static_decode_setup(int dev, const StaticDecodeSetup **out) {
    std::lock_guard<std::mutex> lk(g_static_mu);
    StaticDecodeSetup &s = g_static_setup[dev];
    if (!s.ready) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, lc_static_decode_scratch) != cudaSuccess || !ptr) {
            cudaGetLastError();
            return LC_ERR_CUDA;
        }
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            sms <= 0) {
            cudaGetLastError();
            return LC_ERR_CUDA;
        }
        int rc = static_max_ctas<64>(sms, &s.max_ctas64);
        if (!rc) rc = static_max_ctas<128>(sms, &s.max_ctas128);
        if (rc) return rc;
        s.scratch = ptr;
        s.ready = true;
    }
    *out = &s;
    return LC_OK;
}

template <int HD>
int launch_decode_static(const DecodeParams &prm, int grid, const void *k_pool,
                         const void *v_pool, cudaStream_t stream) {
    CUtensorMap mk, mv;
    int rc = pool_tensor_map_nocache(k_pool, prm.pool_rows, HD, &mk);
    if (rc) return rc;
    rc = pool_tensor_map_nocache(v_pool, prm.pool_rows, HD, &mv);
    if (rc) return rc;
    paged_decode_kernel<HD, false><<<grid, kThreads, DecodeCfg<HD>::kSmemBytes, stream>>>(mk, mv, prm);
    return launch_status();
}

}  // namespace
}  // namespace lc

extern "C" int lc_paged_decode_static(void *out, int64_t out_stride, const void *q,
                                      int64_t q_stride, const void *k_pool, const void *v_pool,
                                      int64_t num_blocks, int num_layers, int layer,
                                      int num_q_heads, int num_kv_heads, int head_dim,
                                      const int *block_tables, int table_stride,
                                      const int *context_lens, int len_offset, int batch,
                                      int max_context_len, int partition_tokens, float sm_scale,
                                      int *dev_status, lc_stream_t stream) {
    if (!out || !q || !k_pool || !v_pool || !block_tables || !context_lens)
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (batch < 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || num_q_heads <= 0 ||
        num_kv_heads <= 0 || num_blocks <= 0 || table_stride <= 0 || len_offset < 0 ||
        len_offset > 1 || partition_tokens < 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if (batch == 0) return LC_OK;
    if (!aligned16(k_pool) || !aligned16(v_pool) || !aligned16(q) || (q_stride & 7) ||
        ((uintptr_t)out & 1))
        return LC_ERR_MISALIGNED;
    if (q_stride < (int64_t)num_q_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim)
        return LC_ERR_INVALID_ARGUMENT;
    const int64_t pool_rows = num_blocks * num_layers * num_kv_heads * kBlockSize;
    if (pool_rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    if (dev < 0 || dev >= kStaticMaxDevices) return LC_ERR_NOT_SUPPORTED;
    const StaticDecodeSetup *setup = nullptr;
    int rc = static_decode_setup(dev, &setup);
    if (rc) return rc;

    const int G = segments_per_seq(num_q_heads, num_kv_heads);
    const int cmax = head_dim == 64 ? setup->max_ctas64 : setup->max_ctas128;
    const WsLayout wl = ws_layout(batch, G, head_dim, cmax);
    if (wl.total() > (size_t)LC_PAGED_DECODE_STATIC_SCRATCH_BYTES)
        return LC_ERR_WORKSPACE_TOO_SMALL;  // batch too large for the fixed scratch
    cudaStream_t s = as_stream(stream);
    // The arrival counters and the tags of the partial words must start at
    // zero. A call that completes leaves them so; one that gave up (timeout)
    // may not, and this entry has no re-initialisation call, so each call
    // clears the part of the scratch it uses.
    if (cudaMemsetAsync(setup->scratch, 0, wl.total(), s) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    int grid = cmax;
    if (max_context_len > 0) {
        const long long pages_hint =
            (long long)batch * G * ((max_context_len + kBlockSize - 1) / kBlockSize);
        const long long want = (pages_hint + kMinPagesPerCta - 1) / kMinPagesPerCta;
        if (want < grid) grid = (int)(want < 1 ? 1 : want);
    }
    DecodeParams prm{};
    prm.out = (bf16 *)out;
    prm.out_stride = out_stride;
    prm.q = (const bf16 *)q;
    prm.q_stride = q_stride;
    prm.tables = block_tables;
    prm.table_stride = table_stride;
    prm.ctx_lens = context_lens;
    prm.len_offset = len_offset;
    prm.batch = batch;
    prm.pool_rows = pool_rows;
    prm.num_blocks = num_blocks;
    prm.num_layers = num_layers;
    prm.layer = layer;
    prm.num_q_heads = num_q_heads;
    prm.num_kv_heads = num_kv_heads;
    prm.group = num_q_heads / num_kv_heads;
    prm.ctas_per_kv = (prm.group + kHeadsPerCta - 1) / kHeadsPerCta;
    prm.seg_per_seq = G;
    prm.partition_tokens = partition_tokens;
    prm.scale_log2 = sm_scale * 1.4426950408889634f;
    uint8_t *ws = (uint8_t *)setup->scratch;
    prm.ws_cnt = (int *)ws;
    prm.ws_lse = (uint64_t *)(ws + wl.cnt_bytes);
    prm.ws_o = (uint64_t *)(ws + wl.cnt_bytes + wl.lse_bytes);
    prm.status = dev_status;
    prm.out_vec = ((uintptr_t)out & 3) == 0 && out_stride % 2 == 0;
    return head_dim == 64 ? launch_decode_static<64>(prm, grid, k_pool, v_pool, s)
                          : launch_decode_static<128>(prm, grid, k_pool, v_pool, s);
}
