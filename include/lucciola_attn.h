/*
 * lucciola_attn.h - C ABI of the B200 (sm_100a) attention hot path of lucciola-rs.
 *
 * The path: bias + rotate-half RoPE on the new token's Q/K, append of K and V+bias
 * into the paged KV pool, paged flash-decoding attention (GQA), and the causal
 * prefill that attends over the same paged pool.
 *
 * Conventions shared by every entry point:
 *   - All tensors are device pointers; bf16 tensors are passed as void*.
 *   - Paged pool layout (unchanged from src/layers/kv_cache.rs:60-68 and
 *     src/kernels/kv_cache.cu:31-48):
 *         k_pool, v_pool : bf16 [num_blocks][num_layers][num_kv_heads][16][head_dim]
 *     A page of one (block, layer, kv_head) is 16 * head_dim contiguous bf16 values.
 *   - Block tables are int32 logical->physical page maps; the batched entry points
 *     take one row per sequence, `table_stride` int32 apart.
 *   - Every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 *     stream), allocates nothing, and performs no host synchronisation, so the calls
 *     can be captured in a CUDA graph.
 *   - Return value: LC_OK or an lc_status code. Argument errors are detected on the
 *     host before anything is launched. Data errors that only the device can see
 *     (a block-table entry outside the pool, a position outside the table) are
 *     recorded as bits in the optional `dev_status` word (int32, device memory):
 *     the offending page is skipped (writes) or read as zeros (attention), never
 *     dereferenced out of bounds.
 *   - head_dim is 64 or 128 and block_size is 16, as in src/kernels.rs:37-47 and
 *     src/layers/kv_cache.rs:35.
 */
#ifndef LUCCIOLA_ATTN_H
#define LUCCIOLA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *lc_stream_t; /* cudaStream_t */

enum lc_status {
    LC_OK = 0,
    LC_ERR_INVALID_ARGUMENT = 1,    /* null pointer, negative or inconsistent size          */
    LC_ERR_UNSUPPORTED_HEAD_DIM = 2,/* head_dim not 64/128 (src/kernels.rs:40-45 bails too) */
    LC_ERR_UNSUPPORTED_SHAPE = 3,   /* block_size != 16, num_q_heads % num_kv_heads != 0     */
    LC_ERR_WORKSPACE_TOO_SMALL = 4, /* workspace smaller than lc_*_workspace_size()          */
    LC_ERR_MISALIGNED = 5,          /* a pool/tensor pointer not 16-byte aligned             */
    LC_ERR_CUDA = 6,                /* a CUDA runtime/driver call failed                     */
    LC_ERR_DEVICE_BOUNDS = 7,       /* device saw an out-of-range page or position           */
    LC_ERR_DEVICE_TIMEOUT = 8,      /* a bounded device-side wait gave up                    */
    LC_ERR_OUT_OF_BLOCKS = 9,       /* KV cache free list exhausted (kv_cache.rs:110-113)    */
    LC_ERR_OUT_OF_MEMORY = 10,      /* KV cache does not fit the memory budget (:40-48)      */
    LC_ERR_NOT_SUPPORTED = 11,      /* no sm_100 device / feature unavailable                */
    LC_ERR_NO_FREE_SLOT = 12        /* lc_kv_pool: every sequence slot is in use             */
};

/* Bits a kernel ORs into the optional device status word. */
#define LC_DEV_BAD_BLOCK 0x1   /* block-table entry outside [0, num_blocks)            */
#define LC_DEV_BAD_POS 0x2     /* position outside the block table or RoPE table       */
#define LC_DEV_TIMEOUT 0x4     /* a pipeline wait exceeded its bound                    */

const char *lc_status_string(int status);
/* Maps a device status word (read back by the caller) to an lc_status code. */
int lc_status_from_device_word(int word);
/* Library version string, e.g. "lucciola-b200 0.1 sm_100a". */
const char *lc_version(void);

/* Programmatic dependent launch for the decode kernels (lc_paged_decode,
 * lc_rope_append_decode, lc_flash_decoding), process-wide:
 *   0 (default) plain launches;
 *   1 launched with programmatic stream serialization: a decode grid may be
 *     scheduled while the preceding grid in the stream retires and waits for
 *     it (griddepcontrol.wait) before reading or writing any memory;
 *   2 as 1, but the grid reads the context lengths and computes its split
 *     before that wait, and lc_rope_append_decode also reads block tables,
 *     the positions, the q/k/v biases and the RoPE cos/sin rows, and starts
 *     loading this layer's cached K/V pages before it; only the qkv rows are
 *     read after it. The kernel launched just before on the same stream must
 *     then not write the context lengths/positions, the block tables, the
 *     biases, the RoPE tables, or this layer's cached K/V (a decode step's QKV
 *     projection or another layer's attention qualifies).
 * Returns the previous mode, or -1 for an invalid mode. */
int lc_set_dependent_launch(int mode);

/* ------------------------------------------------------------------------- */
/* Reference-shaped entry points (single sequence, drop-in for the kernels).  */
/* ------------------------------------------------------------------------- */

/* Replaces `rope` (src/kernels/rope.cu:3-13) as launched by
 * CudaFunctions::apply_rope (src/kernels.rs:203-246). In place:
 *   q[h] <- bf16(rot(q[h] + q_bias[h]))  for h < num_q_heads
 *   k[h] <- bf16(rot(k[h] + k_bias[h]))  for h < num_k_heads
 * with rot = rotate-half over pairs (d, d + head_dim/2) using
 * cos_cache/sin_cache[*pos_ptr][d] (f32 [max_pos][head_dim/2]). Bit-exact. */
int lc_rope(void *q, const void *q_bias, void *k, const void *k_bias,
            const float *cos_cache, const float *sin_cache, const int *pos_ptr,
            int head_dim, int num_q_heads, int num_k_heads, lc_stream_t stream);

/* Replaces `update_kv_cache_kernel` (src/kernels/kv_cache.cu:3-17) as launched
 * by KVCache::update (src/layers/kv_cache.rs:124-173). Writes the token at
 * position *pos_ptr: k_pool <- new_k (bit copy), v_pool <- bf16(new_v + v_bias).
 * `max_seq_len` is accepted and unused, as in the reference. */
int lc_update_kv_cache(void *k_pool, void *v_pool, const void *new_k,
                       const void *new_v, const void *v_bias,
                       const int *block_table, int layer_id, const int *pos_ptr,
                       int num_layers, int num_kv_heads, int max_seq_len,
                       int head_dim, int block_size, lc_stream_t stream);

/* Replaces flash_decoding_kernel_64/128 (src/kernels/attention.cu:178-240) as
 * launched by CudaFunctions::apply_flash_decoding (src/kernels.rs:248-320).
 * Attention of num_q_heads query heads over cache positions 0..=*current_pos.
 * Extra arguments the reference's launch site has but its kernel does not:
 *   host_pos           - the host copy of the position (kernels.rs:258), used
 *                        only to size the grid; the device value decides.
 *   num_physical_blocks- pool size in pages (KVCache::num_physical_blocks).
 *   workspace          - split-K scratch of lc_flash_decoding_workspace_size()
 *                        bytes, zeroed once by lc_paged_decode_workspace_init. */
size_t lc_flash_decoding_workspace_size(int num_q_heads, int head_dim,
                                        int max_seq_len);
int lc_flash_decoding(void *output, const void *q, const void *k_pool,
                      const void *v_pool, const int *block_table, int layer_idx,
                      int num_q_heads, int num_kv_heads, int head_dim,
                      int max_seq_len, const int *current_pos, float sm_scale,
                      int block_size, int num_layers, int host_pos,
                      int64_t num_physical_blocks, void *workspace,
                      size_t workspace_bytes, lc_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Batched entry points (the B200 path).                                     */
/* ------------------------------------------------------------------------- */

/* Fused bias + RoPE + KV append for `num_seqs * tokens_per_seq` token rows
 * (decode: tokens_per_seq = 1; prefill: the prompt). Row r belongs to sequence
 * r / tokens_per_seq and sits at position positions[r]. Each row of `qkv`
 * (`row_stride` bf16 apart) holds [q (Hq*hd) | k (Hkv*hd) | v (Hkv*hd)], the
 * layout of InferenceBuffers::qkv_states (src/layers/buffers.rs:28-31,
 * src/models.rs:495-498). Effects, bit-identical to rope -> update_kv_cache:
 *   q, k rotated in place (bf16), v untouched;
 *   k_pool[page(pos)] <- rotated k,  v_pool[page(pos)] <- bf16(v + v_bias).
 * Biases are bf16 [Hq*hd], [Hkv*hd], [Hkv*hd] (src/models.rs:500-502).
 * rope_rows = rows of the cos/sin tables (positions must be < rope_rows). */
int lc_rope_append(void *qkv, int64_t row_stride, int num_seqs,
                   int tokens_per_seq, const int *positions,
                   const void *q_bias, const void *k_bias, const void *v_bias,
                   const float *cos_cache, const float *sin_cache, int rope_rows,
                   void *k_pool, void *v_pool, int64_t num_blocks,
                   int num_layers, int layer, int num_q_heads, int num_kv_heads,
                   int head_dim, const int *block_tables, int table_stride,
                   int *dev_status, lc_stream_t stream);

/* Split-K workspace for lc_paged_decode on the current device (bytes). It holds
 * one arrival counter per (sequence, kv-head slice) and the fp32 partials of
 * segments split across CTAs; its size depends on the device's SM count (a
 * host-only caller gets the size for a 148-SM B200). */
size_t lc_paged_decode_workspace_size(int batch, int num_q_heads,
                                      int num_kv_heads, int head_dim);
/* Zeroes the workspace (once, after allocation). Every lc_paged_decode call
 * leaves its arrival counters at zero again, except one whose status word
 * reports LC_DEV_TIMEOUT: a launch that gave up may leave counters set, so
 * zero the workspace again before the next call. */
int lc_paged_decode_workspace_init(void *workspace, size_t workspace_bytes,
                                   lc_stream_t stream);

/* Batched paged decode attention. For sequence b with n_b = context_lens[b] +
 * len_offset cached tokens (len_offset = 1 when context_lens holds positions,
 * as the reference's pos_ptr does), every query head h of q (row b, `q_stride`
 * bf16 between rows, heads contiguous) attends over cache tokens 0..n_b-1 of
 * kv head h / (Hq/Hkv):
 *   out[b][h] = softmax_t(q.k_t * sm_scale) . v_t     (fp32 accumulation)
 * out is bf16 [batch][Hq][head_dim] with `out_stride` bf16 between rows.
 * The kernel is persistent: the 16-token pages of all (sequence, kv head)
 * segments are split evenly over the CTAs; split segments are merged with a
 * log-sum-exp reduction. partition_tokens > 0 caps the split at about that
 * many tokens per CTA (0 = fill the GPU). max_context_len is an optional host
 * hint (0 = none) that trims the grid for small batches; lengths are read on
 * the device. With batch 1, partition_tokens 0 and a hint of at least 32
 * tokens the call runs the single-sequence form described at
 * lc_rope_append_decode (thread-block clusters). */
int lc_paged_decode(void *out, int64_t out_stride, const void *q,
                    int64_t q_stride, const void *k_pool, const void *v_pool,
                    int64_t num_blocks, int num_layers, int layer,
                    int num_q_heads, int num_kv_heads, int head_dim,
                    const int *block_tables, int table_stride,
                    const int *context_lens, int len_offset, int batch,
                    int max_context_len, int partition_tokens, float sm_scale,
                    void *workspace, size_t workspace_bytes, int *dev_status,
                    lc_stream_t stream);

/* Fused decode step for a batch: lc_rope_append with one
 * row per sequence followed by lc_paged_decode with len_offset = 1, in ONE
 * launch. For sequence b the new token sits at position positions[b]; its q
 * and k are biased and rotated, its k and v + v_bias are appended to the pools
 * at that position, and the attention covers positions 0..positions[b]
 * inclusive. qkv rows are [q | k | v] (`row_stride` bf16 apart) and are only
 * read: unlike rope (src/kernels/rope.cu:37-53) the rotated q/k are not written
 * back, a side effect nothing after the attention reads (o_proj consumes the
 * attention output, src/models.rs:553-566). Pool writes are bit-identical to
 * lc_rope_append; the output is that of lc_paged_decode. Workspace as for
 * lc_paged_decode (lc_paged_decode_workspace_size).
 * With batch 1, partition_tokens 0 and max_context_len of at least 32 tokens
 * (one sequence, as Qwen2Model::generate decodes, src/models.rs:230-245),
 * each kv head's pages are split over one thread-block cluster of up to 16
 * CTAs whose pieces are combined in shared memory; max_context_len then sizes
 * the clusters, so it should be the real length or close above it. The
 * workspace is passed as always and left as found. */
int lc_rope_append_decode(void *out, int64_t out_stride, const void *qkv,
                          int64_t row_stride, const int *positions,
                          const void *q_bias, const void *k_bias,
                          const void *v_bias, const float *cos_cache,
                          const float *sin_cache, int rope_rows, void *k_pool,
                          void *v_pool, int64_t num_blocks, int num_layers,
                          int layer, int num_q_heads, int num_kv_heads,
                          int head_dim, const int *block_tables,
                          int table_stride, int batch, int max_context_len,
                          int partition_tokens, float sm_scale, void *workspace,
                          size_t workspace_bytes, int *dev_status,
                          lc_stream_t stream);

/* lc_rope_append_decode with an input gate: the launch reads its qkv rows only
 * once the int at `gate` (device-visible memory) is non-zero, waiting for it
 * on the device (2 s at most, then LC_DEV_TIMEOUT in the status word). For a
 * step whose rows arrive by a host-to-device copy on another stream that then
 * sets the gate (a 4-byte copy after the rows' copy, in the same stream): the
 * decode launches need no cross-stream dependency, which would cost each one
 * its programmatic overlap with the launch before. The caller clears the gate
 * before the next use. out may be mapped pinned host memory (the outputs then
 * cross PCIe as they are written). */
int lc_rope_append_decode_gated(void *out, int64_t out_stride, const void *qkv,
                                int64_t row_stride, const int *positions, const void *q_bias,
                                const void *k_bias, const void *v_bias, const float *cos_cache,
                                const float *sin_cache, int rope_rows, void *k_pool,
                                void *v_pool, int64_t num_blocks, int num_layers, int layer,
                                int num_q_heads, int num_kv_heads, int head_dim,
                                const int *block_tables, int table_stride, int batch,
                                int max_context_len, int partition_tokens, float sm_scale,
                                void *workspace, size_t workspace_bytes, int *dev_status,
                                const int *gate, lc_stream_t stream);

/* Allocation-free variant of lc_paged_decode. No counterpart in the reference.
 * For callers that cannot allocate device memory while they decode (a serving
 * loop that must not call cudaMalloc/cudaFree because they may synchronise the
 * device, or a host whose device memory is all reserved for its own pools):
 * the split-K scratch is a fixed array of LC_PAGED_DECODE_STATIC_SCRATCH_BYTES
 * that the library keeps on every GPU it is loaded on, until the process exits.
 * Same arguments and results as lc_paged_decode, minus the workspace.
 *   - The first call on a device sets it up (resolves the array's device
 *     address, sets kernel attributes); make that first call before any CUDA
 *     stream capture on that device.
 *   - Returns LC_ERR_WORKSPACE_TOO_SMALL, launching nothing, when the batch
 *     needs more scratch than the fixed size (lc_paged_decode_workspace_size
 *     tells how much a shape needs).
 *   - Every call uses the same array: calls that may run at the same time on
 *     the GPU (different streams) race; order them on one stream.
 *   - Allocates nothing: no cudaMalloc/cudaFree, no host allocation. */
#define LC_PAGED_DECODE_STATIC_SCRATCH_BYTES (8u << 20)
int lc_paged_decode_static(void *out, int64_t out_stride, const void *q,
                           int64_t q_stride, const void *k_pool,
                           const void *v_pool, int64_t num_blocks,
                           int num_layers, int layer, int num_q_heads,
                           int num_kv_heads, int head_dim,
                           const int *block_tables, int table_stride,
                           const int *context_lens, int len_offset, int batch,
                           int max_context_len, int partition_tokens,
                           float sm_scale, int *dev_status, lc_stream_t stream);

/* How lc_proj_gemm / lc_qkv_proj_rope_append run a decode step (M <= 128 token
 * rows: one per sequence) on the current device: the weights are split into
 * ceil(N / 128)-row tiles, each tile's K over a cluster of `split` CTAs;
 * `ctas` is the grid, and (optional) `clusters_that_fit` how many clusters of
 * that size the device runs at once and `ctas_per_sm` how many of the
 * kernel's CTAs share an SM. No counterpart in the reference, which calls
 * cublasGemmEx (src/models.rs:252-292). */
int lc_proj_decode_plan(int N, int K, int *split, int *ctas, int *clusters_that_fit,
                        int *ctas_per_sm);

/* Causal prefill over the paged pool (tcgen05 tensor-core path). Query token i
 * of sequence b sits at position start_pos[b] + i and attends to cache tokens
 * 0..=start_pos[b]+i of its kv head; the K/V of the prompt must already be in
 * the pool (lc_rope_append). q and out are [num_seqs*tokens_per_seq] rows of
 * Hq*head_dim bf16, `q_stride` / `out_stride` apart. The reference runs this
 * as tokens_per_seq sequential decode steps (src/models.rs:486-550). */
int lc_paged_prefill(void *out, int64_t out_stride, const void *q,
                     int64_t q_stride, const void *k_pool, const void *v_pool,
                     int64_t num_blocks, int num_layers, int layer,
                     int num_q_heads, int num_kv_heads, int head_dim,
                     const int *block_tables, int table_stride,
                     const int *start_pos, int num_seqs, int tokens_per_seq,
                     int max_start_pos, float sm_scale, int *dev_status,
                     lc_stream_t stream);

/* Copies the cached K/V of every sequence into dense bf16
 * [batch][max_context_len][Hkv][head_dim] tensors through the block tables
 * (the same page addressing the attention kernels use; rows >= n_b untouched). */
int lc_gather_kv(void *k_out, void *v_out, const void *k_pool,
                 const void *v_pool, int64_t num_blocks, int num_layers,
                 int layer, int num_kv_heads, int head_dim,
                 const int *block_tables, int table_stride,
                 const int *context_lens, int len_offset, int batch,
                 int max_context_len, int *dev_status, lc_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Host-side mirror of the reference's Rust layer API (owning objects).       */
/* ------------------------------------------------------------------------- */

/* RopeCache::new (src/layers/rope.rs:10-40): f32 cos/sin [max_pos][hd/2],
 * theta = (pos / scale) / base^(2i/hd); scale_factor <= 0 means none.
 * lc_rope_table_host fills caller-provided host arrays (no GPU). */
void lc_rope_table_host(int max_position_embeddings, int head_dim, float base,
                        float scale_factor, float *cos_out, float *sin_out);
typedef struct lc_rope_cache lc_rope_cache;
int lc_rope_cache_new(int max_position_embeddings, int head_dim, float base,
                      float scale_factor, lc_stream_t stream,
                      lc_rope_cache **out);
const float *lc_rope_cache_cos(const lc_rope_cache *rc);
const float *lc_rope_cache_sin(const lc_rope_cache *rc);
void lc_rope_cache_free(lc_rope_cache *rc);

/* KVCache (src/layers/kv_cache.rs:12-174). Pool blocks =
 * min(budget / bytes_per_block, ceil(max_position_embeddings / 16)) where
 * budget = total * memory_fraction - used (kv_cache.rs:37-59). Free list is
 * LIFO so blocks come out 0, 1, 2, ... (kv_cache.rs:73-76). */
typedef struct lc_kv_cache lc_kv_cache;
int lc_kv_cache_new(int num_hidden_layers, int num_attention_heads,
                    int num_key_value_heads, int head_dim,
                    int max_position_embeddings, float memory_fraction,
                    lc_stream_t stream, lc_kv_cache **out);
/* KVCache::prepare_for_step (kv_cache.rs:106-122). Unlike the reference, which
 * pushes at most one block per call, this pushes blocks until the table covers
 * `pos`; for consecutive positions the two are identical. */
int lc_kv_cache_prepare_for_step(lc_kv_cache *c, lc_stream_t stream, int pos);
/* KVCache::update (kv_cache.rs:124-173): prepare_for_step + append launch. */
int lc_kv_cache_update(lc_kv_cache *c, lc_stream_t stream, int layer_idx,
                       int pos, const int *pos_ptr, const void *k_input,
                       const void *v_input, const void *v_bias);
void *lc_kv_cache_k_pool(lc_kv_cache *c);
void *lc_kv_cache_v_pool(lc_kv_cache *c);
int *lc_kv_cache_block_table(lc_kv_cache *c);
int64_t lc_kv_cache_num_physical_blocks(const lc_kv_cache *c);
int lc_kv_cache_max_seq_len(const lc_kv_cache *c);
int lc_kv_cache_num_allocated_blocks(const lc_kv_cache *c);
void lc_kv_cache_free(lc_kv_cache *c);

/* CudaFunctions::apply_flash_decoding (src/kernels.rs:248-320) over an
 * lc_kv_cache: scale = 1/sqrt(head_dim) as in kernels.rs:264, workspace owned
 * by the cache object. */
int lc_apply_flash_decoding(lc_kv_cache *c, lc_stream_t stream, void *output,
                            const void *q, int layer_idx, int pos,
                            const int *pos_ptr, int num_q_heads);

/* ------------------------------------------------------------------------- */
/* Projections either side of attention (tcgen05 tensor cores).               */
/* ------------------------------------------------------------------------- */
/* out[M][N] = x[M][K] . w[N][K]^T, fp32 accumulation, bf16 result: what
 * Qwen2Model::matmul_bf16 computes with cublasGemmEx (src/models.rs:252-292).
 * residual == NULL is beta 0 (qkv_proj, models.rs:470-483); otherwise
 * out = bf16(acc + residual) (o_proj with beta 1 into hidden_states,
 * models.rs:553-566; residual may be out). Row-major with row strides in
 * elements; N % 32 == 0, K % 8 == 0, pointers 16-byte aligned, strides
 * multiples of 8. */
int lc_proj_gemm(void *out, int64_t out_stride, const void *x, int64_t x_stride,
                 const void *w, int64_t w_stride, int M, int N, int K,
                 const void *residual, int64_t res_stride, lc_stream_t stream);

/* The QKV projection of a prompt with lc_rope_append fused into its epilogue:
 * qkv[t] = x[t] . w_qkv^T (N = (Hq + 2 Hkv) * head_dim, K = hidden) rounded to
 * bf16, then q and k biased and rotated in place and k / v + bias appended to
 * the pools, exactly as lc_rope_append over the same rows (arguments as
 * there). The rows, pools and status are bit-identical to lc_proj_gemm
 * followed by lc_rope_append. */
int lc_qkv_proj_rope_append(void *qkv, int64_t row_stride, const void *x, int64_t x_stride,
                            const void *w_qkv, int64_t w_stride, int hidden, int num_seqs,
                            int tokens_per_seq, const int *positions, const void *q_bias,
                            const void *k_bias, const void *v_bias, const float *cos_cache,
                            const float *sin_cache, int rope_rows, void *k_pool, void *v_pool,
                            int64_t num_blocks, int num_layers, int layer, int num_q_heads,
                            int num_kv_heads, int head_dim, const int *block_tables,
                            int table_stride, int *dev_status, lc_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Token selection from the logits of a batch of sequences.                   */
/* ------------------------------------------------------------------------- */
/* Greedy: out_idx[b] = index of the largest logit of row b (rows of `vocab`
 * bf16, row_stride elements apart), as CudaFunctions::apply_argmax /
 * argmax_kernel (src/kernels.rs:322-344, src/kernels/sampling.cu) chooses it,
 * ties included (lower i % 1024, then lower i); 0xffffffff when no logit
 * exceeds -1e30. One launch for the whole batch; any row stride. */
int lc_argmax(const void *logits, int64_t row_stride, int vocab, int batch, unsigned *out_idx,
              lc_stream_t stream);

/* Bytes of candidates lc_sample_top_p keeps per call: batch * n * 8, with
 * n = 32 * (top_k / 32); 0 for an unsupported top_k. Layout: int32 keys
 * [batch][n], then float values [batch][n], each row partition-major as the
 * reference's top_k_filter writes its candidates. */
size_t lc_sample_workspace_size(int batch, int top_k);

/* Top-k / top-p sampling, as CudaFunctions::apply_sort_and_sample
 * (src/kernels.rs:346-490, src/kernels/sampling_optimized.cu) for each row b:
 * the top_k / 32 largest logits of each of 32 vocabulary partitions, sorted
 * (descending, the reference's bitonic network), softmax over them, the
 * smallest prefix whose probability reaches top_p[b], and the candidate whose
 * cumulative interval holds rand_vals[b] * that prefix's probability (device
 * arrays of `batch` floats; the reference draws rand_val on the host per
 * step). n = 32 * (top_k / 32) must be a power of two from 32 to 1024
 * (LC_ERR_UNSUPPORTED_SHAPE otherwise, as the reference bails), vocab >= 32.
 * The candidate set is exact; the draw equals the reference's except where
 * rand * cutoff falls within fp32 rounding of a cumulative boundary. When no
 * candidate wins (rounding at the top) out_idx[b] is left as it was, as in the
 * reference. Two launches for the whole batch. */
int lc_sample_top_p(const void *logits, int64_t row_stride, int vocab, int batch, int top_k,
                    const float *top_p, const float *rand_vals, unsigned *out_idx,
                    void *workspace, size_t workspace_bytes, lc_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Batched token-step driver: many sequences in one paged pool.               */
/* ------------------------------------------------------------------------- */
/* The reference's KVCache holds one sequence (one block table,
 * kv_cache.rs:12-174) and its decode loop steps one token of one sequence
 * (models.rs:230-245, attention section :486-550). lc_kv_pool is the batched
 * replacement of that part: one K and one V pool of num_blocks 16-token pages
 * ([num_blocks][num_layers][num_kv_heads][16][head_dim] bf16, zeroed) shared
 * by up to max_seqs sequences, each owning a list of pages; one LIFO free list
 * (a fresh pool hands out pages 0, 1, 2, ... as kv_cache.rs:73-76 does).
 *
 * lc_block_alloc is its page bookkeeping alone, in host memory. */
typedef struct lc_block_alloc lc_block_alloc;
int lc_block_alloc_new(int64_t num_blocks, int max_seqs, int max_blocks_per_seq,
                       lc_block_alloc **out);
/* Takes the lowest free slot (LC_ERR_NO_FREE_SLOT when none). */
int lc_block_alloc_add_seq(lc_block_alloc *a, int *slot);
/* Returns the slot's pages to the free list (handed out again in the same
 * order) and frees the slot. */
int lc_block_alloc_release_seq(lc_block_alloc *a, int slot);
/* Grows the slot's page list to cover `tokens` tokens. LC_ERR_OUT_OF_BLOCKS
 * when the free list cannot (nothing is taken then); LC_ERR_INVALID_ARGUMENT
 * beyond max_blocks_per_seq pages. */
int lc_block_alloc_reserve(lc_block_alloc *a, int slot, int tokens);
/* Copies up to `capacity` of the slot's pages (logical order) to dst and
 * returns how many it has (-1 for a bad slot). */
int lc_block_alloc_row(const lc_block_alloc *a, int slot, int *dst, int capacity);
int64_t lc_block_alloc_num_free(const lc_block_alloc *a);
/* 64-bit hash of the whole bookkeeping state (slots, page lists, free list in
 * hand-out order). Ranks that shard a model by kv head keep one pool each with
 * identical block tables by issuing the same add/reserve/release calls; equal
 * fingerprints (one all-reduce of a word) confirm that they still agree. */
uint64_t lc_block_alloc_fingerprint(const lc_block_alloc *a);
void lc_block_alloc_free(lc_block_alloc *a);

/* Pool capacity as KVCache::new sizes it (src/layers/kv_cache.rs:37-59):
 * budget = total * memory_fraction (f32) - (total - free) bytes, over the K+V
 * bytes of one 16-token page of every layer (2 * L * Hkv * 16 * hd * 2). Unlike
 * the reference there is no cap at one sequence's pages (the pool is shared);
 * the result is capped so that pool rows fit an int32 index, and is 0 when
 * the budget is not above what is already used. Pure arithmetic, no device. */
int64_t lc_kv_pool_blocks_for_budget(int num_layers, int num_kv_heads, int head_dim,
                                     uint64_t free_bytes, uint64_t total_bytes,
                                     float memory_fraction);
/* The same with free/total from cudaMemGetInfo on the current device;
 * LC_ERR_OUT_OF_MEMORY when no page fits. Head-sharded ranks pass their local
 * kv-head count. */
int lc_kv_pool_capacity(int num_layers, int num_kv_heads, int head_dim, float memory_fraction,
                        int64_t *num_blocks);

/* The device pool. max_seq_len bounds every sequence (table rows of
 * ceil(max_seq_len / 16) entries). Creation allocates and zeroes everything it
 * needs (pools, the step's tables and positions, the split-K workspace, pinned
 * staging); the step calls below allocate nothing. */
typedef struct lc_kv_pool lc_kv_pool;
int lc_kv_pool_new(int num_layers, int num_q_heads, int num_kv_heads, int head_dim,
                   int max_seqs, int max_seq_len, int64_t num_blocks,
                   lc_stream_t stream, lc_kv_pool **out);
int lc_kv_pool_add_sequence(lc_kv_pool *p, int *slot);
int lc_kv_pool_release_sequence(lc_kv_pool *p, int slot);
/* One decode step of `batch` distinct sequences: slots[b] is the sequence of
 * batch row b and positions[b] (host) the position of its new token. Pages are
 * reserved to cover positions[b] + 1 tokens, and the step's block tables (batch
 * order) and positions are copied to the pool's device buffers on `stream`.
 * Those buffers keep their addresses, so the per-layer launches of a step may
 * be captured once in a CUDA graph and replayed after each prepare_step with
 * the same batch size. On LC_ERR_OUT_OF_BLOCKS the sequences before the one
 * that failed keep the pages they were given (they need them next step as
 * well) and nothing is uploaded. */
int lc_kv_pool_prepare_step(lc_kv_pool *p, lc_stream_t stream, int batch,
                            const int *slots, const int *positions);
/* Layer `layer` of the prepared step: bias + RoPE + append of each row's new
 * token and attention over its sequence (lc_rope_append_decode, scale
 * 1/sqrt(head_dim)). qkv rows [q | k | v] in batch order; out [batch][Hq*hd]. */
int lc_kv_pool_decode_layer(lc_kv_pool *p, lc_stream_t stream, int layer, void *out,
                            int64_t out_stride, const void *qkv, int64_t row_stride,
                            const void *q_bias, const void *k_bias, const void *v_bias,
                            const float *cos_cache, const float *sin_cache, int rope_rows,
                            int *dev_status);
/* A prompt of `tokens` tokens of sequence `slot` at positions start_pos.. :
 * reserves its pages and uploads its table row and positions. */
int lc_kv_pool_prepare_prefill(lc_kv_pool *p, lc_stream_t stream, int slot, int start_pos,
                               int tokens);
/* Layer `layer` of the prepared prompt: lc_rope_append over its qkv rows (q and
 * k rotated in place, K/V appended), then lc_paged_prefill into out. */
int lc_kv_pool_prefill_layer(lc_kv_pool *p, lc_stream_t stream, int layer, void *out,
                             int64_t out_stride, void *qkv, int64_t row_stride,
                             const void *q_bias, const void *k_bias, const void *v_bias,
                             const float *cos_cache, const float *sin_cache, int rope_rows,
                             int *dev_status);
void *lc_kv_pool_k_pool(lc_kv_pool *p);
void *lc_kv_pool_v_pool(lc_kv_pool *p);
const int *lc_kv_pool_step_tables(const lc_kv_pool *p);
const int *lc_kv_pool_step_positions(const lc_kv_pool *p);
int lc_kv_pool_table_stride(const lc_kv_pool *p);
int64_t lc_kv_pool_num_blocks(const lc_kv_pool *p);
int64_t lc_kv_pool_num_free_blocks(const lc_kv_pool *p);
int lc_kv_pool_sequence_pages(const lc_kv_pool *p, int slot, int *dst, int capacity);
/* After a decode layer whose status word reported LC_DEV_TIMEOUT: zeroes the
 * pool's split-K workspace on `stream` (see lc_paged_decode_workspace_init). */
int lc_kv_pool_recover(lc_kv_pool *p, lc_stream_t stream);
/* lc_block_alloc_fingerprint of the pool's page bookkeeping. */
uint64_t lc_kv_pool_fingerprint(const lc_kv_pool *p);
void lc_kv_pool_free(lc_kv_pool *p);

/* ------------------------------------------------------------------------- */
/* Multi-GPU host logic.                                                      */
/* ------------------------------------------------------------------------- */

/* Sequence sharding: assigns each of `batch` sequences to one of `num_ranks`
 * ranks by longest-processing-time-first bin packing on context length
 * (ties by index). rank_of[b] receives the rank. Deterministic. */
int lc_shard_sequences(const int *context_lens, int batch, int num_ranks,
                       int *rank_of);
/* KV-head sharding: rank r owns kv heads [r*Hkv/R, (r+1)*Hkv/R) and q heads
 * [r*Hq/R, (r+1)*Hq/R). Writes first kv head and count; fails unless R | Hkv. */
int lc_shard_kv_heads(int num_q_heads, int num_kv_heads, int num_ranks,
                      int rank, int *first_kv_head, int *num_local_kv_heads);

/* ------------------------------------------------------------------------- */
/* Peer exchange: KV-head-sharded decode that writes every rank's output.    */
/* No counterpart in the reference (one GPU, src/models.rs:486-550).         */
/* ------------------------------------------------------------------------- */

/* Under KV-head sharding each rank computes the attention rows of its own q
 * heads; the next operator (o_proj) wants all heads of every sequence. In
 * place of an all-gather after the decode, lc_rope_append_decode_peer stores
 * each finished output row into the same place of every rank's output buffer
 * (NVLink peer stores from the decode's epilogue), and lc_peer_wait, on each
 * rank, waits on the device until every peer's decode of the same layer has
 * landed.
 *
 * Every rank allocates one exchange region of the same size
 * (lc_peer_region_alloc): its first LC_PEER_SIGNAL_BYTES hold the signal
 * words; output buffers are carved from the rest at the same offsets on every
 * rank. The regions' IPC handles are exchanged by the caller (any host
 * collective) and opened by lc_peer_group_open. One process per GPU; a group
 * holds at most LC_PEER_MAX_RANKS ranks. */
#define LC_PEER_MAX_RANKS 8
#define LC_PEER_SIGNAL_BYTES 256
#define LC_PEER_HANDLE_BYTES 64 /* sizeof(cudaIpcMemHandle_t) */

typedef struct lc_peer_group lc_peer_group;

/* Allocates and zeroes `bytes` (> LC_PEER_SIGNAL_BYTES) of device memory on the
 * current device and writes its IPC handle (LC_PEER_HANDLE_BYTES) to
 * handle_out. */
int lc_peer_region_alloc(size_t bytes, void **region, void *handle_out);
int lc_peer_region_free(void *region);

/* Group of `world` ranks; `region` is this rank's, handles[r *
 * LC_PEER_HANDLE_BYTES] rank r's (this rank's entry is not read). Opens every
 * peer's region in this process (peer access over NVLink). Every region,
 * this rank's and each opened peer's, must hold at least region_bytes from its
 * start (checked against the allocation's extent); otherwise nothing stays
 * open and LC_ERR_INVALID_ARGUMENT is returned. */
int lc_peer_group_open(int rank, int world, void *region, size_t region_bytes,
                       const void *handles, lc_peer_group **out);
/* The same over regions this process already addresses (regions[r] for rank r;
 * several ranks driven from one process, e.g. on one GPU), each checked for
 * region_bytes of room in the same way. */
int lc_peer_group_local(int rank, int world, void *const *regions, size_t region_bytes,
                        lc_peer_group **out);
/* Closes the opened peer mappings; the regions stay allocated. */
void lc_peer_group_destroy(lc_peer_group *g);

/* lc_rope_append_decode whose output rows also land in every peer's region:
 * `out` must lie in this rank's region past the signal words (rows up to
 * batch-1 included), and is written at the same offset in each peer's region.
 * After its last store the launch raises this rank's signal word in every
 * peer's region (system-scope release); a batch of 0 still launches, so that it
 * still signals. Launches and lc_peer_wait calls pair up in order: the k-th
 * wait on a rank waits for the k-th peer decode launch of every other rank of
 * the group. */
int lc_rope_append_decode_peer(void *out, int64_t out_stride, const void *qkv,
                               int64_t row_stride, const int *positions, const void *q_bias,
                               const void *k_bias, const void *v_bias, const float *cos_cache,
                               const float *sin_cache, int rope_rows, void *k_pool,
                               void *v_pool, int64_t num_blocks, int num_layers, int layer,
                               int num_q_heads, int num_kv_heads, int head_dim,
                               const int *block_tables, int table_stride, int batch,
                               int max_context_len, int partition_tokens, float sm_scale,
                               void *workspace, size_t workspace_bytes, int *dev_status,
                               const lc_peer_group *group, lc_stream_t stream);

/* Waits on the device, in stream order after this rank's peer decode launch,
 * until every other rank of the group has signalled the same launch count;
 * launches after it on `stream` see all ranks' rows. A wait that exceeds 2 s
 * sets LC_DEV_TIMEOUT in *dev_status (if given) and returns. */
int lc_peer_wait(const lc_peer_group *group, int *dev_status, lc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LUCCIOLA_ATTN_H */
