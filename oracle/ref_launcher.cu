/*
 * ref_launcher.cu - host launcher for the reference's own CUDA kernels.
 *
 * TEST INFRASTRUCTURE ONLY: the GPU oracle and the reference arm of bench.py.
 * oracle/Makefile compiles this file with -I pointing at the reference's
 * src/kernels directory, so the three reference kernels below are built from
 * their unchanged sources where they lie; nothing of them is copied here. The
 * launch shapes restate the reference's Rust launch code:
 *   rope                    src/kernels.rs:217-218 (cudarc for_num_elems:
 *                           1024-thread blocks, ceil(n/1024) blocks)
 *   update_kv_cache_kernel  src/layers/kv_cache.rs:138-142 (grid Hkv, block hd)
 *   flash_decoding_kernel_* src/kernels.rs:263-284 (grid Hq, block 1024,
 *                           dynamic shared memory formula)
 * Batched and prefill helpers loop over sequences/tokens on the host, one
 * launch each, as src/models.rs:486-550 does for one sequence.
 */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "rope.cu"
#include "kv_cache.cu"
#include "attention.cu"

typedef __nv_bfloat16 bf16;

static int ref_err(cudaError_t e) { return e == cudaSuccess ? 0 : 1000 + (int)e; }

/* RopeCache::new (src/layers/rope.rs:20-31) on the host: t = pos / scale,
 * theta = t / base^((2i)/hd), cos/sin tables f32 [max_pos][hd/2]. Lets the
 * reference arm of bench.py build its tables without the product library. */
extern "C" void ref_rope_table(int max_pos, int head_dim, float base, float scale_factor,
                               float *cos_out, float *sin_out) {
    const int half = head_dim / 2;
    const float scale = scale_factor > 0.0f ? scale_factor : 1.0f;
    for (int pos = 0; pos < max_pos; ++pos)
        for (int i = 0; i < half; ++i) {
            float t = (float)pos / scale;
            float theta = t / powf(base, (float)(2 * i) / (float)head_dim);
            cos_out[(int64_t)pos * half + i] = cosf(theta);
            sin_out[(int64_t)pos * half + i] = sinf(theta);
        }
}

extern "C" int ref_rope(void *q, const void *q_bias, void *k, const void *k_bias,
                        const float *cos_cache, const float *sin_cache,
                        const int *pos_ptr, int head_dim, int num_q_heads,
                        int num_k_heads, cudaStream_t stream) {
    unsigned n = (unsigned)(num_q_heads * (head_dim / 2));
    dim3 grid((n + 1023) / 1024), block(1024);
    rope<<<grid, block, 0, stream>>>((bf16 *)q, (const bf16 *)q_bias, (bf16 *)k,
                                     (const bf16 *)k_bias, cos_cache, sin_cache,
                                     pos_ptr, head_dim, num_q_heads, num_k_heads);
    return ref_err(cudaGetLastError());
}

extern "C" int ref_update_kv_cache(void *k_pool, void *v_pool, const void *new_k,
                                   const void *new_v, const void *v_bias,
                                   const int *block_table, int layer_id,
                                   const int *pos_ptr, int num_layers,
                                   int num_kv_heads, int max_seq_len,
                                   int head_dim, int block_size,
                                   cudaStream_t stream) {
    update_kv_cache_kernel<<<num_kv_heads, head_dim, 0, stream>>>(
        (bf16 *)k_pool, (bf16 *)v_pool, (const bf16 *)new_k, (const bf16 *)new_v,
        (const bf16 *)v_bias, block_table, layer_id, pos_ptr, num_layers,
        num_kv_heads, max_seq_len, head_dim, block_size);
    return ref_err(cudaGetLastError());
}

extern "C" int ref_flash_decoding(void *out, const void *q, const void *k_pool,
                                  const void *v_pool, const int *block_table,
                                  int layer_idx, int num_q_heads,
                                  int num_kv_heads, int head_dim,
                                  int max_seq_len, const int *pos_ptr,
                                  int host_pos, int block_size, int num_layers,
                                  cudaStream_t stream) {
    float scale = 1.0f / sqrtf((float)head_dim);               /* kernels.rs:264 */
    size_t nblk = (size_t)(host_pos + block_size) / block_size; /* :266 */
    const size_t warps = 32;
    size_t smem = head_dim * 4 + nblk * 4 + warps * head_dim * 4 + warps * 4 +
                  warps * 4 + 256;                               /* :272-278 */
    if (smem > 48 * 1024) return 2; /* the reference launches without an opt-in */
    if (head_dim == 64) {
        flash_decoding_kernel_64<<<num_q_heads, 1024, smem, stream>>>(
            (bf16 *)out, (const bf16 *)q, (const bf16 *)k_pool, (const bf16 *)v_pool,
            block_table, layer_idx, num_q_heads, num_kv_heads, head_dim, max_seq_len,
            pos_ptr, scale, block_size, num_layers);
    } else if (head_dim == 128) {
        flash_decoding_kernel_128<<<num_q_heads, 1024, smem, stream>>>(
            (bf16 *)out, (const bf16 *)q, (const bf16 *)k_pool, (const bf16 *)v_pool,
            block_table, layer_idx, num_q_heads, num_kv_heads, head_dim, max_seq_len,
            pos_ptr, scale, block_size, num_layers);
    } else {
        return 3; /* kernels.rs:40-45 */
    }
    return ref_err(cudaGetLastError());
}

/* One decode step for a batch: per sequence b, flash-decoding with table row b
 * and the device position pos_dev[b] (host copy host_pos[b] sizes shared memory). */
extern "C" int ref_paged_decode(void *out, int64_t out_stride, const void *q,
                                int64_t q_stride, const void *k_pool,
                                const void *v_pool, int num_layers, int layer,
                                int num_q_heads, int num_kv_heads, int head_dim,
                                const int *block_tables, int table_stride,
                                const int *pos_dev, const int *host_pos,
                                int batch, int max_seq_len, cudaStream_t stream) {
    for (int b = 0; b < batch; ++b) {
        int rc = ref_flash_decoding((bf16 *)out + (int64_t)b * out_stride,
                                    (const bf16 *)q + (int64_t)b * q_stride, k_pool,
                                    v_pool, block_tables + (int64_t)b * table_stride,
                                    layer, num_q_heads, num_kv_heads, head_dim,
                                    max_seq_len, pos_dev + b, host_pos[b], 16,
                                    num_layers, stream);
        if (rc) return rc;
    }
    return 0;
}

/* Per token row r (sequence r / tokens_per_seq, position pos_dev[r]): rope on
 * the row's q/k, then the append of k and v+bias (src/models.rs:506-534). */
extern "C" int ref_rope_append(void *qkv, int64_t row_stride, int num_seqs,
                               int tokens_per_seq, const int *pos_dev,
                               const void *q_bias, const void *k_bias,
                               const void *v_bias, const float *cos_cache,
                               const float *sin_cache, void *k_pool,
                               void *v_pool, int num_layers, int layer,
                               int num_q_heads, int num_kv_heads, int head_dim,
                               const int *block_tables, int table_stride,
                               int max_seq_len, cudaStream_t stream) {
    int rows = num_seqs * tokens_per_seq;
    for (int r = 0; r < rows; ++r) {
        int b = r / tokens_per_seq;
        bf16 *row = (bf16 *)qkv + (int64_t)r * row_stride;
        bf16 *qp = row;
        bf16 *kp = row + num_q_heads * head_dim;
        bf16 *vp = kp + num_kv_heads * head_dim;
        int rc = ref_rope(qp, q_bias, kp, k_bias, cos_cache, sin_cache, pos_dev + r,
                          head_dim, num_q_heads, num_kv_heads, stream);
        if (rc) return rc;
        rc = ref_update_kv_cache(k_pool, v_pool, kp, vp, v_bias,
                                 block_tables + (int64_t)b * table_stride, layer,
                                 pos_dev + r, num_layers, num_kv_heads, max_seq_len,
                                 head_dim, 16, stream);
        if (rc) return rc;
    }
    return 0;
}

/* The reference's prefill (src/models.rs:486-550): for every token, rope, append,
 * then decode attention over 0..=pos, strictly in order. q rows live in qkv. */
extern "C" int ref_prefill(void *out, int64_t out_stride, void *qkv,
                           int64_t row_stride, int num_seqs, int tokens_per_seq,
                           const int *pos_dev, const int *host_pos,
                           const void *q_bias, const void *k_bias,
                           const void *v_bias, const float *cos_cache,
                           const float *sin_cache, void *k_pool, void *v_pool,
                           int num_layers, int layer, int num_q_heads,
                           int num_kv_heads, int head_dim,
                           const int *block_tables, int table_stride,
                           int max_seq_len, cudaStream_t stream) {
    int rows = num_seqs * tokens_per_seq;
    for (int r = 0; r < rows; ++r) {
        int b = r / tokens_per_seq;
        bf16 *row = (bf16 *)qkv + (int64_t)r * row_stride;
        bf16 *qp = row;
        bf16 *kp = row + num_q_heads * head_dim;
        bf16 *vp = kp + num_kv_heads * head_dim;
        const int *table = block_tables + (int64_t)b * table_stride;
        int rc = ref_rope(qp, q_bias, kp, k_bias, cos_cache, sin_cache, pos_dev + r,
                          head_dim, num_q_heads, num_kv_heads, stream);
        if (!rc)
            rc = ref_update_kv_cache(k_pool, v_pool, kp, vp, v_bias, table, layer,
                                     pos_dev + r, num_layers, num_kv_heads,
                                     max_seq_len, head_dim, 16, stream);
        if (!rc)
            rc = ref_flash_decoding((bf16 *)out + (int64_t)r * out_stride, qp, k_pool,
                                    v_pool, table, layer, num_q_heads, num_kv_heads,
                                    head_dim, max_seq_len, pos_dev + r, host_pos[r],
                                    16, num_layers, stream);
        if (rc) return rc;
    }
    return 0;
}
