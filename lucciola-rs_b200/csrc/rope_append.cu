// rope_append.cu - fused bias + rotate-half RoPE + paged KV append.
//
// One kernel serves three entry points:
//   lc_rope            rotate q (and k) of one token in place     (src/kernels/rope.cu:3-54)
//   lc_update_kv_cache append one token's k and v+bias           (src/kernels/kv_cache.cu:3-59)
//   lc_rope_append     both, for a batch of token rows, one launch (src/models.rs:506-534)
//
// Bit-exactness: the rotate-half arithmetic (rope_math.cuh) rounds as the
// reference kernel does; the q+bias and v+bias additions are single fp32 adds;
// results round to bf16 with RNE.
#include <climits>

#include "lc_common.cuh"
#include "lc_host.h"
#include "rope_math.cuh"

namespace lc {
namespace {

struct RopeAppendParams {
    bf16 *q;        // row 0 of q (rotated in place when rope_q_heads > 0)
    bf16 *k;        // row 0 of k (rotated in place when rope_k_heads > 0)
    const bf16 *v;  // row 0 of v
    int64_t row_stride;
    int rows, tokens_per_seq;
    const int *positions;  // [rows]
    const bf16 *q_bias, *k_bias, *v_bias;
    const float *cos_t, *sin_t;
    int rope_rows;  // < 0: unchecked
    int rope_q_heads, rope_k_heads;
    int append;
    bf16 *k_pool, *v_pool;
    int64_t num_blocks;  // < 0: unchecked
    int num_layers, layer, num_kv_heads, head_dim;
    const int *tables;
    int table_stride;  // <= 0: unchecked
    int *status;
};

// Returns the pool element offset of (pos, kv head 0) for row `row`, or -1 when
// the row must not be appended (status bits set for bad positions/blocks).
__device__ __forceinline__ int64_t append_base(const RopeAppendParams &p, int row, int pos) {
    const int b = row / p.tokens_per_seq;
    const int logical = pos / kBlockSize;
    if (p.table_stride > 0 && logical >= p.table_stride) {
        set_status(p.status, LC_DEV_BAD_POS);
        return -1;
    }
    const int phys = p.tables[(int64_t)b * (p.table_stride > 0 ? p.table_stride : 0) + logical];
    if (p.num_blocks >= 0 && (phys < 0 || phys >= p.num_blocks)) {
        set_status(p.status, LC_DEV_BAD_BLOCK);
        return -1;
    }
    return page_row(phys, p.layer, 0, p.num_layers, p.num_kv_heads) * p.head_dim +
           (int64_t)(pos % kBlockSize) * p.head_dim;
}

// Items of one row: [0, A) rotate pair (head, d) of q (+ k for head < rope_k_heads,
// + append of the rotated k when appending); [A, A+B) append pair (kv head, d) of v
// (+ k as-is when k is not rotated). A = rope_q_heads*half, B = append ? Hkv*half : 0.
__global__ void __launch_bounds__(256) rope_append_kernel(RopeAppendParams p) {
    const int half = p.head_dim >> 1;
    const int items_a = p.rope_q_heads * half;
    const int items_b = p.append ? p.num_kv_heads * half : 0;
    const int per_row = items_a + items_b;
    const int64_t total = (int64_t)p.rows * per_row;
    const int64_t stride_blk = (int64_t)kBlockSize * p.head_dim;  // between kv heads of a page
    for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < total;
         gi += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(gi / per_row);
        const int item = (int)(gi - (int64_t)row * per_row);
        const int pos = p.positions[row];
        if (pos < 0) {
            if (item == 0) set_status(p.status, LC_DEV_BAD_POS);
            continue;
        }
        const int64_t roff = (int64_t)row * p.row_stride;
        if (item < items_a) {
            const int head = item / half, d = item - (item / half) * half;
            if (p.rope_rows >= 0 && pos >= p.rope_rows) {
                if (item == 0) set_status(p.status, LC_DEV_BAD_POS);
                continue;
            }
            const float c = p.cos_t[(int64_t)pos * half + d];
            const float s = p.sin_t[(int64_t)pos * half + d];
            const int i1 = head * p.head_dim + d, i2 = i1 + half;
            bf16 *q = p.q + roff;
            const float v1 = __fadd_rn(__bfloat162float(q[i1]), __bfloat162float(p.q_bias[i1]));
            const float v2 = __fadd_rn(__bfloat162float(q[i2]), __bfloat162float(p.q_bias[i2]));
            q[i1] = __float2bfloat16(rot_sub(v1, c, v2, s));
            q[i2] = __float2bfloat16(rot_add(v1, s, v2, c));
            if (head < p.rope_k_heads) {
                bf16 *k = p.k + roff;
                const float k1 = __fadd_rn(__bfloat162float(k[i1]), __bfloat162float(p.k_bias[i1]));
                const float k2 = __fadd_rn(__bfloat162float(k[i2]), __bfloat162float(p.k_bias[i2]));
                const bf16 r1 = __float2bfloat16(rot_sub(k1, c, k2, s));
                const bf16 r2 = __float2bfloat16(rot_add(k1, s, k2, c));
                k[i1] = r1;
                k[i2] = r2;
                if (p.append) {
                    const int64_t base = append_base(p, row, pos);
                    if (base >= 0) {
                        bf16 *dst = p.k_pool + base + head * stride_blk;
                        dst[d] = r1;
                        dst[d + half] = r2;
                    }
                }
            }
        } else {
            const int j = item - items_a;
            const int head = j / half, d = j - (j / half) * half;
            const int64_t base = append_base(p, row, pos);
            if (base < 0) continue;
            const int i1 = head * p.head_dim + d, i2 = i1 + half;
            const bf16 *v = p.v + roff;
            const int64_t o = base + head * stride_blk;
            p.v_pool[o + d] =
                __float2bfloat16(__fadd_rn(__bfloat162float(v[i1]), __bfloat162float(p.v_bias[i1])));
            p.v_pool[o + d + half] =
                __float2bfloat16(__fadd_rn(__bfloat162float(v[i2]), __bfloat162float(p.v_bias[i2])));
            if (p.rope_k_heads == 0) {
                const bf16 *k = p.k + roff;
                p.k_pool[o + d] = k[i1];
                p.k_pool[o + d + half] = k[i2];
            }
        }
    }
}

// 8 consecutive bf16 (16 bytes) as floats, and back with RNE rounding.
__device__ __forceinline__ void load8(const bf16 *src, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4 *>(src);
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __low2float(h[i]);
        f[2 * i + 1] = __high2float(h[i]);
    }
}
__device__ __forceinline__ void store8(bf16 *dst, const float (&f)[8]) {
    uint4 u;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4 *>(dst) = u;
}
__device__ __forceinline__ void load8f(const float *src, float (&f)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(src)[0];
    const float4 b = reinterpret_cast<const float4 *>(src)[1];
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
}

// The same items with eight dims each (16-byte loads and stores), for callers
// whose rows, biases, RoPE tables and pools are 16-byte aligned: item (head,
// chunk) covers dims [8 chunk, 8 chunk + 8) of the first half and their
// partners in the second. Per element the arithmetic is that of the kernel
// above.
__global__ void __launch_bounds__(256) rope_append_vec_kernel(RopeAppendParams p) {
    const int half = p.head_dim >> 1;
    const int cph = half >> 3;  // chunks of 8 dims per half
    const int items_a = p.rope_q_heads * cph;
    const int items_b = p.append ? p.num_kv_heads * cph : 0;
    const int per_row = items_a + items_b;
    const int64_t total = (int64_t)p.rows * per_row;
    const int64_t stride_blk = (int64_t)kBlockSize * p.head_dim;  // between kv heads of a page
    for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < total;
         gi += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(gi / per_row);
        const int item = (int)(gi - (int64_t)row * per_row);
        const int pos = p.positions[row];
        if (pos < 0) {
            if (item == 0) set_status(p.status, LC_DEV_BAD_POS);
            continue;
        }
        const int64_t roff = (int64_t)row * p.row_stride;
        if (item < items_a) {
            const int head = item / cph, d = (item - head * cph) * 8;
            if (p.rope_rows >= 0 && pos >= p.rope_rows) {
                if (item == 0) set_status(p.status, LC_DEV_BAD_POS);
                continue;
            }
            float c[8], sn[8], x1[8], x2[8], b1[8], b2[8];
            load8f(p.cos_t + (int64_t)pos * half + d, c);
            load8f(p.sin_t + (int64_t)pos * half + d, sn);
            const int i1 = head * p.head_dim + d, i2 = i1 + half;
            bf16 *q = p.q + roff;
            load8(q + i1, x1);
            load8(q + i2, x2);
            load8(p.q_bias + i1, b1);
            load8(p.q_bias + i2, b2);
            float o1[8], o2[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float v1 = __fadd_rn(x1[e], b1[e]), v2 = __fadd_rn(x2[e], b2[e]);
                o1[e] = rot_sub(v1, c[e], v2, sn[e]);
                o2[e] = rot_add(v1, sn[e], v2, c[e]);
            }
            store8(q + i1, o1);
            store8(q + i2, o2);
            if (head < p.rope_k_heads) {
                bf16 *k = p.k + roff;
                load8(k + i1, x1);
                load8(k + i2, x2);
                load8(p.k_bias + i1, b1);
                load8(p.k_bias + i2, b2);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float k1 = __fadd_rn(x1[e], b1[e]), k2 = __fadd_rn(x2[e], b2[e]);
                    o1[e] = rot_sub(k1, c[e], k2, sn[e]);
                    o2[e] = rot_add(k1, sn[e], k2, c[e]);
                }
                store8(k + i1, o1);
                store8(k + i2, o2);
                if (p.append) {
                    const int64_t base = append_base(p, row, pos);
                    if (base >= 0) {
                        bf16 *dst = p.k_pool + base + head * stride_blk;
                        store8(dst + d, o1);
                        store8(dst + d + half, o2);
                    }
                }
            }
        } else {
            const int j = item - items_a;
            const int head = j / cph, d = (j - head * cph) * 8;
            const int64_t base = append_base(p, row, pos);
            if (base < 0) continue;
            const int i1 = head * p.head_dim + d, i2 = i1 + half;
            const bf16 *v = p.v + roff;
            const int64_t o = base + head * stride_blk;
            float x1[8], x2[8], b1[8], b2[8];
            load8(v + i1, x1);
            load8(v + i2, x2);
            load8(p.v_bias + i1, b1);
            load8(p.v_bias + i2, b2);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                x1[e] = __fadd_rn(x1[e], b1[e]);
                x2[e] = __fadd_rn(x2[e], b2[e]);
            }
            store8(p.v_pool + o + d, x1);
            store8(p.v_pool + o + d + half, x2);
            if (p.rope_k_heads == 0) {
                const bf16 *k = p.k + roff;
                *reinterpret_cast<uint4 *>(p.k_pool + o + d) = *reinterpret_cast<const uint4 *>(k + i1);
                *reinterpret_cast<uint4 *>(p.k_pool + o + d + half) =
                    *reinterpret_cast<const uint4 *>(k + i2);
            }
        }
    }
}

bool vec_ok(const RopeAppendParams &p) {
    auto a16 = [](const void *x) { return !x || ((uintptr_t)x & 15) == 0; };
    return (p.head_dim & 15) == 0 && (p.row_stride & 7) == 0 && a16(p.q) && a16(p.k) &&
           a16(p.v) && a16(p.q_bias) && a16(p.k_bias) && a16(p.v_bias) && a16(p.cos_t) &&
           a16(p.sin_t) && a16(p.k_pool) && a16(p.v_pool);
}

int launch(const RopeAppendParams &p, cudaStream_t stream) {
    const int threads = 256;
    const int64_t cap = (int64_t)sm_count() * 16;
    if (vec_ok(p)) {
        const int cph = p.head_dim / 16;
        const int64_t per_row =
            (int64_t)p.rope_q_heads * cph + (p.append ? (int64_t)p.num_kv_heads * cph : 0);
        const int64_t total = per_row * p.rows;
        if (total == 0) return LC_OK;
        int64_t blocks = (total + threads - 1) / threads;
        if (blocks > cap) blocks = cap;
        rope_append_vec_kernel<<<(unsigned)blocks, threads, 0, stream>>>(p);
        return launch_status();
    }
    const int half = p.head_dim / 2;
    const int64_t per_row =
        (int64_t)p.rope_q_heads * half + (p.append ? (int64_t)p.num_kv_heads * half : 0);
    const int64_t total = per_row * p.rows;
    if (total == 0) return LC_OK;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > cap) blocks = cap;
    rope_append_kernel<<<(unsigned)blocks, threads, 0, stream>>>(p);
    return launch_status();
}

bool head_dim_ok(int hd) { return hd == 64 || hd == 128; }

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" int lc_rope(void *q, const void *q_bias, void *k, const void *k_bias,
                       const float *cos_cache, const float *sin_cache, const int *pos_ptr,
                       int head_dim, int num_q_heads, int num_k_heads, lc_stream_t stream) {
    if (!q || !q_bias || !cos_cache || !sin_cache || !pos_ptr) return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads <= 0 || num_k_heads < 0 || head_dim <= 0 || (head_dim & 1))
        return LC_ERR_INVALID_ARGUMENT;
    if (num_k_heads > 0 && (!k || !k_bias)) return LC_ERR_INVALID_ARGUMENT;
    RopeAppendParams p{};
    p.q = (bf16 *)q;
    p.k = (bf16 *)k;
    p.row_stride = 0;
    p.rows = 1;
    p.tokens_per_seq = 1;
    p.positions = pos_ptr;
    p.q_bias = (const bf16 *)q_bias;
    p.k_bias = (const bf16 *)k_bias;
    p.cos_t = cos_cache;
    p.sin_t = sin_cache;
    p.rope_rows = -1;
    p.rope_q_heads = num_q_heads;
    // rope.cu:42 rotates k for head < num_k_heads among the q-head threads only.
    p.rope_k_heads = num_k_heads < num_q_heads ? num_k_heads : num_q_heads;
    p.append = 0;
    p.head_dim = head_dim;
    p.num_kv_heads = num_k_heads;
    return launch(p, as_stream(stream));
}

extern "C" int lc_update_kv_cache(void *k_pool, void *v_pool, const void *new_k,
                                  const void *new_v, const void *v_bias,
                                  const int *block_table, int layer_id, const int *pos_ptr,
                                  int num_layers, int num_kv_heads, int max_seq_len,
                                  int head_dim, int block_size, lc_stream_t stream) {
    (void)max_seq_len;  // unused by the reference kernel as well (kv_cache.cu:14)
    if (!k_pool || !v_pool || !new_k || !new_v || !v_bias || !block_table || !pos_ptr)
        return LC_ERR_INVALID_ARGUMENT;
    if (block_size != kBlockSize) return LC_ERR_UNSUPPORTED_SHAPE;
    if (num_layers <= 0 || num_kv_heads <= 0 || layer_id < 0 || layer_id >= num_layers ||
        head_dim <= 0 || (head_dim & 1))
        return LC_ERR_INVALID_ARGUMENT;
    RopeAppendParams p{};
    p.k = (bf16 *)new_k;
    p.v = (const bf16 *)new_v;
    p.rows = 1;
    p.tokens_per_seq = 1;
    p.positions = pos_ptr;
    p.v_bias = (const bf16 *)v_bias;
    p.rope_rows = -1;
    p.append = 1;
    p.k_pool = (bf16 *)k_pool;
    p.v_pool = (bf16 *)v_pool;
    p.num_blocks = -1;
    p.num_layers = num_layers;
    p.layer = layer_id;
    p.num_kv_heads = num_kv_heads;
    p.head_dim = head_dim;
    p.tables = block_table;
    p.table_stride = 0;
    return launch(p, as_stream(stream));
}

extern "C" int lc_rope_append(void *qkv, int64_t row_stride, int num_seqs, int tokens_per_seq,
                              const int *positions, const void *q_bias, const void *k_bias,
                              const void *v_bias, const float *cos_cache,
                              const float *sin_cache, int rope_rows, void *k_pool,
                              void *v_pool, int64_t num_blocks, int num_layers, int layer,
                              int num_q_heads, int num_kv_heads, int head_dim,
                              const int *block_tables, int table_stride, int *dev_status,
                              lc_stream_t stream) {
    if (!qkv || !positions || !q_bias || !k_bias || !v_bias || !cos_cache || !sin_cache ||
        !k_pool || !v_pool || !block_tables)
        return LC_ERR_INVALID_ARGUMENT;
    if (!head_dim_ok(head_dim)) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (num_seqs < 0 || tokens_per_seq <= 0 || num_layers <= 0 || layer < 0 ||
        layer >= num_layers || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
        table_stride <= 0 || rope_rows <= 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if (row_stride < (int64_t)(num_q_heads + 2 * num_kv_heads) * head_dim)
        return LC_ERR_INVALID_ARGUMENT;
    if ((int64_t)num_seqs * tokens_per_seq > INT_MAX) return LC_ERR_INVALID_ARGUMENT;
    RopeAppendParams p{};
    p.q = (bf16 *)qkv;
    p.k = p.q + (int64_t)num_q_heads * head_dim;
    p.v = p.k + (int64_t)num_kv_heads * head_dim;
    p.row_stride = row_stride;
    p.rows = num_seqs * tokens_per_seq;
    p.tokens_per_seq = tokens_per_seq;
    p.positions = positions;
    p.q_bias = (const bf16 *)q_bias;
    p.k_bias = (const bf16 *)k_bias;
    p.v_bias = (const bf16 *)v_bias;
    p.cos_t = cos_cache;
    p.sin_t = sin_cache;
    p.rope_rows = rope_rows;
    p.rope_q_heads = num_q_heads;
    p.rope_k_heads = num_kv_heads;
    p.append = 1;
    p.k_pool = (bf16 *)k_pool;
    p.v_pool = (bf16 *)v_pool;
    p.num_blocks = num_blocks;
    p.num_layers = num_layers;
    p.layer = layer;
    p.num_kv_heads = num_kv_heads;
    p.head_dim = head_dim;
    p.tables = block_tables;
    p.table_stride = table_stride;
    p.status = dev_status;
    return launch(p, as_stream(stream));
}
