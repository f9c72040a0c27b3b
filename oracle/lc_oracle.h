/*
 * lc_oracle.h - CPU restatement of lucciola-rs's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the parity tests, smoke() and
 * bench.py's CPU-baseline leg compare against; the product library never links
 * or calls it. Every function follows a reference kernel statement by statement
 * (file:line cited per function) in plain scalar C with fp32 arithmetic.
 *
 * Parity pin: the reference ships no tests, fixtures or golden vectors. The
 * restatement is pinned against outputs of the reference's own CUDA kernels
 * (compiled unchanged from src/kernels/{rope,kv_cache,attention}.cu into
 * oracle/_ref by oracle/Makefile) recorded on a B200 as fixtures under
 * tests/golden/ by tests/golden/make_golden.py.
 *
 * bf16 values are uint16_t bit patterns; conversion to bf16 is round to
 * nearest even, as __float2bfloat16 and the `half` crate do.
 */
#ifndef LC_ORACLE_H
#define LC_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float lco_bf16_to_f32(uint16_t h);
uint16_t lco_f32_to_bf16(float f);

/* src/layers/rope.rs:23-31 */
void lco_rope_table(int max_pos, int head_dim, float base, float scale_factor,
                    float *cos_out, float *sin_out);

/* Contraction modes for the two rotate-half expressions of src/kernels/rope.cu:37-38
 * (x1*c - x2*s and x1*s + x2*c): 0 = two rounded products, 1 = fma on the first
 * product (fma(x1,c,-(x2*s)), fma(x1,s,x2*c)), 2 = fma on the second product. */
void lco_rope(uint16_t *q, const uint16_t *q_bias, uint16_t *k,
              const uint16_t *k_bias, const float *cos_cache,
              const float *sin_cache, int pos, int head_dim, int num_q_heads,
              int num_k_heads, int sub_mode, int add_mode);

/* src/kernels/kv_cache.cu:18-58 */
void lco_update_kv_cache(uint16_t *k_pool, uint16_t *v_pool,
                         const uint16_t *new_k, const uint16_t *new_v,
                         const uint16_t *v_bias, const int *block_table,
                         int layer_id, int pos, int num_layers,
                         int num_kv_heads, int head_dim, int block_size);

/* src/kernels/attention.cu:20-175 with its 32-warp x 32-lane structure
 * (launch shape from src/kernels.rs:268-284). Returns 0, or -1 when a
 * block-table entry is outside [0, num_blocks). */
int lco_flash_decoding(uint16_t *out, const uint16_t *q, const uint16_t *k_pool,
                       const uint16_t *v_pool, const int *block_table,
                       int layer_idx, int num_q_heads, int num_kv_heads,
                       int head_dim, int pos, float sm_scale, int block_size,
                       int num_layers, int64_t num_blocks);

/* Batched decode: lco_flash_decoding per sequence b with table row b and
 * pos = context_lens[b] + len_offset - 1 (models.rs:536-549 per sequence).
 * Runs on `num_threads` POSIX threads split over sequences. */
int lco_paged_decode(uint16_t *out, int64_t out_stride, const uint16_t *q,
                     int64_t q_stride, const uint16_t *k_pool,
                     const uint16_t *v_pool, int64_t num_blocks, int num_layers,
                     int layer, int num_q_heads, int num_kv_heads, int head_dim,
                     const int *block_tables, int table_stride,
                     const int *context_lens, int len_offset, int batch,
                     float sm_scale, int num_threads);

/* rope -> update_kv_cache per row, in the order of src/models.rs:506-534. */
int lco_rope_append(uint16_t *qkv, int64_t row_stride, int num_seqs,
                    int tokens_per_seq, const int *positions,
                    const uint16_t *q_bias, const uint16_t *k_bias,
                    const uint16_t *v_bias, const float *cos_cache,
                    const float *sin_cache, uint16_t *k_pool, uint16_t *v_pool,
                    int num_layers, int layer, int num_q_heads,
                    int num_kv_heads, int head_dim, const int *block_tables,
                    int table_stride, int sub_mode, int add_mode);

/* Causal prefill as the reference runs it (src/models.rs:486-550): token t of
 * sequence b attends over positions 0..=start_pos[b]+t by one
 * lco_flash_decoding call per token. The pool must already hold the K/V. */
int lco_paged_prefill(uint16_t *out, int64_t out_stride, const uint16_t *q,
                      int64_t q_stride, const uint16_t *k_pool,
                      const uint16_t *v_pool, int64_t num_blocks,
                      int num_layers, int layer, int num_q_heads,
                      int num_kv_heads, int head_dim, const int *block_tables,
                      int table_stride, const int *start_pos, int num_seqs,
                      int tokens_per_seq, float sm_scale, int num_threads);

/* Dense copy of the paged K/V through the tables: [batch][max_ctx][Hkv][hd]. */
int lco_gather_kv(uint16_t *k_out, uint16_t *v_out, const uint16_t *k_pool,
                  const uint16_t *v_pool, int64_t num_blocks, int num_layers,
                  int layer, int num_kv_heads, int head_dim,
                  const int *block_tables, int table_stride,
                  const int *context_lens, int len_offset, int batch,
                  int max_context_len);

/* Token selection (src/kernels/sampling.cu, sampling_optimized.cu). */
int lco_argmax(const uint16_t *logits, int vocab);
void lco_top_k_filter(const uint16_t *logits, int vocab, int kpb, int *keys, float *values);
int lco_top_p_sample(const int *keys, const float *values, int n, float top_p, float rand_val,
                     double *margin);

#ifdef __cplusplus
}
#endif
#endif
