/*
 * lc_oracle.c - CPU restatement of lucciola-rs's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see lc_oracle.h): used by tests/, smoke() and the
 * CPU-baseline leg of bench.py, never by the product library.
 *
 * Compiled with -ffp-contract=off: every place where the reference's CUDA
 * compiler contracts a multiply-add into an FMA (NVRTC's default fmad=true)
 * is written here as an explicit fmaf(), everything else rounds per operation.
 */
#include "lc_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

float lco_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t lco_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff; /* NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                     /* round to nearest even */
    return (uint16_t)(u >> 16);
}

/* src/layers/rope.rs:23-31: t = pos / scale; theta = t / base^((2i)/hd). */
void lco_rope_table(int max_pos, int head_dim, float base, float scale_factor,
                    float *cos_out, float *sin_out) {
    const int half = head_dim / 2;
    const float scale = scale_factor > 0.0f ? scale_factor : 1.0f;
    for (int pos = 0; pos < max_pos; ++pos) {
        for (int i = 0; i < half; ++i) {
            float t = (float)pos / scale;
            float theta = t / powf(base, (float)(2 * i) / (float)head_dim);
            cos_out[(int64_t)pos * half + i] = cosf(theta);
            sin_out[(int64_t)pos * half + i] = sinf(theta);
        }
    }
}

static float rot_sub(float x1, float c, float x2, float s, int mode) {
    if (mode == 1) return fmaf(x1, c, -(x2 * s));
    if (mode == 2) return fmaf(-x2, s, x1 * c);
    return x1 * c - x2 * s;
}

static float rot_add(float x1, float s, float x2, float c, int mode) {
    if (mode == 1) return fmaf(x1, s, x2 * c);
    if (mode == 2) return fmaf(x2, c, x1 * s);
    return x1 * s + x2 * c;
}

/* src/kernels/rope.cu:14-53: one "thread" per (q head, d < hd/2). */
void lco_rope(uint16_t *q, const uint16_t *q_bias, uint16_t *k,
              const uint16_t *k_bias, const float *cos_cache,
              const float *sin_cache, int pos, int head_dim, int num_q_heads,
              int num_k_heads, int sub_mode, int add_mode) {
    const int half = head_dim / 2;
    for (int i = 0; i < num_q_heads * half; ++i) {
        int head = i / half, d = i % half;
        float c = cos_cache[(int64_t)pos * half + d];
        float s = sin_cache[(int64_t)pos * half + d];
        int i1 = head * head_dim + d, i2 = i1 + half;
        float v1 = lco_bf16_to_f32(q[i1]) + lco_bf16_to_f32(q_bias[i1]);
        float v2 = lco_bf16_to_f32(q[i2]) + lco_bf16_to_f32(q_bias[i2]);
        q[i1] = lco_f32_to_bf16(rot_sub(v1, c, v2, s, sub_mode));
        q[i2] = lco_f32_to_bf16(rot_add(v1, s, v2, c, add_mode));
        if (head < num_k_heads) {
            float k1 = lco_bf16_to_f32(k[i1]) + lco_bf16_to_f32(k_bias[i1]);
            float k2 = lco_bf16_to_f32(k[i2]) + lco_bf16_to_f32(k_bias[i2]);
            k[i1] = lco_f32_to_bf16(rot_sub(k1, c, k2, s, sub_mode));
            k[i2] = lco_f32_to_bf16(rot_add(k1, s, k2, c, add_mode));
        }
    }
}

/* Element offset of (physical block, layer, kv head, token in block) in a pool
 * laid out [blocks][layers][kv_heads][block_size][head_dim]
 * (src/kernels/kv_cache.cu:39-48, src/kernels/attention.cu:71-87). */
static int64_t pool_offset(int64_t phys, int layer, int head, int tok,
                           int num_layers, int num_kv_heads, int block_size,
                           int head_dim) {
    int64_t stride_block = (int64_t)num_layers * num_kv_heads * block_size * head_dim;
    int64_t stride_layer = (int64_t)num_kv_heads * block_size * head_dim;
    int64_t stride_head = (int64_t)block_size * head_dim;
    return phys * stride_block + (int64_t)layer * stride_layer +
           (int64_t)head * stride_head + (int64_t)tok * head_dim;
}

/* src/kernels/kv_cache.cu:18-58 */
void lco_update_kv_cache(uint16_t *k_pool, uint16_t *v_pool,
                         const uint16_t *new_k, const uint16_t *new_v,
                         const uint16_t *v_bias, const int *block_table,
                         int layer_id, int pos, int num_layers,
                         int num_kv_heads, int head_dim, int block_size) {
    int phys = block_table[pos / block_size];
    int off_in_block = pos % block_size;
    for (int h = 0; h < num_kv_heads; ++h) {
        int64_t base = pool_offset(phys, layer_id, h, off_in_block, num_layers,
                                   num_kv_heads, block_size, head_dim);
        for (int d = 0; d < head_dim; ++d) {
            int idx = h * head_dim + d;
            k_pool[base + d] = new_k[idx];
            float vv = lco_bf16_to_f32(new_v[idx]) + lco_bf16_to_f32(v_bias[idx]);
            v_pool[base + d] = lco_f32_to_bf16(vv);
        }
    }
}

#define REF_WARPS 32 /* blockDim 1024 (src/kernels.rs:268, 280-284) */
#define REF_LANES 32

/* src/kernels/attention.cu:20-175, one call per query head group of the grid. */
int lco_flash_decoding(uint16_t *out, const uint16_t *q, const uint16_t *k_pool,
                       const uint16_t *v_pool, const int *block_table,
                       int layer_idx, int num_q_heads, int num_kv_heads,
                       int head_dim, int pos, float sm_scale, int block_size,
                       int num_layers, int64_t num_blocks) {
    const int per_lane = head_dim / REF_LANES; /* local_o slots used (:65-68) */
    int nblk = (pos + block_size) / block_size;  /* :35 */
    for (int b = 0; b < nblk; ++b)
        if (block_table[b] < 0 || block_table[b] >= num_blocks) return -1;

    float s_q[128];
    float red_m[REF_WARPS], red_l[REF_WARPS];
    float red_o[REF_WARPS][128];
    for (int qh = 0; qh < num_q_heads; ++qh) {
        int kvh = qh / (num_q_heads / num_kv_heads); /* :23 */
        for (int i = 0; i < head_dim; ++i) s_q[i] = lco_bf16_to_f32(q[qh * head_dim + i]);

        for (int w = 0; w < REF_WARPS; ++w) {
            float local_m = -1e20f, local_l = 0.0f;   /* :61-62 */
            float local_o[REF_LANES][4];
            memset(local_o, 0, sizeof(local_o));
            for (int t = w; t <= pos; t += REF_WARPS) { /* :80 */
                int64_t base = pool_offset(block_table[t / block_size], layer_idx,
                                           kvh, t % block_size, num_layers,
                                           num_kv_heads, block_size, head_dim);
                /* :90-96, lane-strided dot with contraction into fma */
                float lane_score[REF_LANES];
                for (int lane = 0; lane < REF_LANES; ++lane) {
                    float sc = 0.0f;
                    for (int i = lane; i < head_dim; i += REF_LANES)
                        sc = fmaf(s_q[i], lco_bf16_to_f32(k_pool[base + i]), sc);
                    lane_score[lane] = sc;
                }
                /* :99-102, __shfl_down_sync tree; lane 0's value is broadcast */
                for (int off = 16; off > 0; off /= 2) {
                    float nxt[REF_LANES];
                    for (int lane = 0; lane < REF_LANES; ++lane)
                        nxt[lane] = lane_score[lane] +
                                    (lane + off < REF_LANES ? lane_score[lane + off]
                                                            : lane_score[lane]);
                    memcpy(lane_score, nxt, sizeof(nxt));
                }
                float score = lane_score[0] * sm_scale; /* :103 */
                /* :106-111 */
                float m_prev = local_m;
                local_m = fmaxf(m_prev, score);
                float exp_m = expf(m_prev - local_m);
                float exp_s = expf(score - local_m);
                local_l = fmaf(local_l, exp_m, exp_s);
                /* :114-119 */
                for (int lane = 0; lane < REF_LANES; ++lane) {
                    int idx = 0;
                    for (int i = lane; i < head_dim; i += REF_LANES, ++idx) {
                        float vv = lco_bf16_to_f32(v_pool[base + i]);
                        local_o[lane][idx] = fmaf(local_o[lane][idx], exp_m, vv * exp_s);
                    }
                }
            }
            red_m[w] = local_m; /* :124-135 */
            red_l[w] = local_l;
            for (int lane = 0; lane < REF_LANES; ++lane) {
                int idx = 0;
                for (int i = lane; i < head_dim; i += REF_LANES, ++idx)
                    red_o[w][i] = local_o[lane][idx];
            }
        }
        (void)per_lane;
        /* :140-174 warp-0 merge */
        float global_m = -1e20f;
        for (int w = 0; w < REF_WARPS; ++w) global_m = fmaxf(global_m, red_m[w]);
        float global_l = 0.0f;
        for (int w = 0; w < REF_WARPS; ++w) {
            float diff = red_m[w] - global_m;
            if (red_m[w] <= -1e19f) continue;
            global_l = fmaf(red_l[w], expf(diff), global_l);
        }
        for (int i = 0; i < head_dim; ++i) {
            float sum_o = 0.0f;
            for (int w = 0; w < REF_WARPS; ++w) {
                if (red_m[w] <= -1e19f) continue;
                float scale = expf(red_m[w] - global_m);
                sum_o = fmaf(red_o[w][i], scale, sum_o);
            }
            sum_o /= global_l;
            out[qh * head_dim + i] = lco_f32_to_bf16(sum_o);
        }
    }
    return 0;
}

typedef struct {
    uint16_t *out;
    int64_t out_stride;
    const uint16_t *q;
    int64_t q_stride;
    const uint16_t *k_pool, *v_pool;
    int64_t num_blocks;
    int num_layers, layer, num_q_heads, num_kv_heads, head_dim;
    const int *block_tables;
    int table_stride;
    const int *context_lens; /* decode: lengths; prefill: start positions */
    int len_offset, batch, tokens_per_seq, prefill;
    float sm_scale;
    int next;                /* work counter (protected by mu) */
    int err;
    pthread_mutex_t mu;
} decode_job;

static void run_item(decode_job *j, int item) {
    int b = j->prefill ? item / j->tokens_per_seq : item;
    int t = j->prefill ? item % j->tokens_per_seq : 0;
    int pos = j->prefill ? j->context_lens[b] + t
                         : j->context_lens[b] + j->len_offset - 1;
    int64_t row = j->prefill ? (int64_t)item : (int64_t)b;
    if (pos < 0) { /* empty context: defined as a zero output */
        memset(j->out + row * j->out_stride, 0,
               sizeof(uint16_t) * j->num_q_heads * j->head_dim);
        return;
    }
    int rc = lco_flash_decoding(j->out + row * j->out_stride, j->q + row * j->q_stride,
                                j->k_pool, j->v_pool,
                                j->block_tables + (int64_t)b * j->table_stride,
                                j->layer, j->num_q_heads, j->num_kv_heads,
                                j->head_dim, pos, j->sm_scale, 16, j->num_layers,
                                j->num_blocks);
    if (rc) {
        pthread_mutex_lock(&j->mu);
        j->err = rc;
        pthread_mutex_unlock(&j->mu);
    }
}

static void *decode_worker(void *arg) {
    decode_job *j = (decode_job *)arg;
    int total = j->prefill ? j->batch * j->tokens_per_seq : j->batch;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        int item = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (item >= total) break;
        run_item(j, item);
    }
    return NULL;
}

static int run_job(decode_job *j, int num_threads) {
    if (num_threads < 1) num_threads = 1;
    if (num_threads > 256) num_threads = 256;
    pthread_mutex_init(&j->mu, NULL);
    j->next = 0;
    j->err = 0;
    pthread_t th[256];
    for (int i = 1; i < num_threads; ++i) pthread_create(&th[i], NULL, decode_worker, j);
    decode_worker(j);
    for (int i = 1; i < num_threads; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&j->mu);
    return j->err;
}

int lco_paged_decode(uint16_t *out, int64_t out_stride, const uint16_t *q,
                     int64_t q_stride, const uint16_t *k_pool,
                     const uint16_t *v_pool, int64_t num_blocks, int num_layers,
                     int layer, int num_q_heads, int num_kv_heads, int head_dim,
                     const int *block_tables, int table_stride,
                     const int *context_lens, int len_offset, int batch,
                     float sm_scale, int num_threads) {
    decode_job j;
    memset(&j, 0, sizeof(j));
    j.out = out; j.out_stride = out_stride; j.q = q; j.q_stride = q_stride;
    j.k_pool = k_pool; j.v_pool = v_pool; j.num_blocks = num_blocks;
    j.num_layers = num_layers; j.layer = layer; j.num_q_heads = num_q_heads;
    j.num_kv_heads = num_kv_heads; j.head_dim = head_dim;
    j.block_tables = block_tables; j.table_stride = table_stride;
    j.context_lens = context_lens; j.len_offset = len_offset; j.batch = batch;
    j.tokens_per_seq = 1; j.prefill = 0; j.sm_scale = sm_scale;
    return run_job(&j, num_threads);
}

int lco_paged_prefill(uint16_t *out, int64_t out_stride, const uint16_t *q,
                      int64_t q_stride, const uint16_t *k_pool,
                      const uint16_t *v_pool, int64_t num_blocks,
                      int num_layers, int layer, int num_q_heads,
                      int num_kv_heads, int head_dim, const int *block_tables,
                      int table_stride, const int *start_pos, int num_seqs,
                      int tokens_per_seq, float sm_scale, int num_threads) {
    decode_job j;
    memset(&j, 0, sizeof(j));
    j.out = out; j.out_stride = out_stride; j.q = q; j.q_stride = q_stride;
    j.k_pool = k_pool; j.v_pool = v_pool; j.num_blocks = num_blocks;
    j.num_layers = num_layers; j.layer = layer; j.num_q_heads = num_q_heads;
    j.num_kv_heads = num_kv_heads; j.head_dim = head_dim;
    j.block_tables = block_tables; j.table_stride = table_stride;
    j.context_lens = start_pos; j.batch = num_seqs;
    j.tokens_per_seq = tokens_per_seq; j.prefill = 1; j.sm_scale = sm_scale;
    return run_job(&j, num_threads);
}

/* src/models.rs:486-534: per token row, rope (rope.cu) then append (kv_cache.cu). */
int lco_rope_append(uint16_t *qkv, int64_t row_stride, int num_seqs,
                    int tokens_per_seq, const int *positions,
                    const uint16_t *q_bias, const uint16_t *k_bias,
                    const uint16_t *v_bias, const float *cos_cache,
                    const float *sin_cache, uint16_t *k_pool, uint16_t *v_pool,
                    int num_layers, int layer, int num_q_heads,
                    int num_kv_heads, int head_dim, const int *block_tables,
                    int table_stride, int sub_mode, int add_mode) {
    int rows = num_seqs * tokens_per_seq;
    for (int r = 0; r < rows; ++r) {
        int b = r / tokens_per_seq;
        uint16_t *row = qkv + (int64_t)r * row_stride;
        uint16_t *qp = row;
        uint16_t *kp = row + num_q_heads * head_dim;
        uint16_t *vp = kp + num_kv_heads * head_dim;
        lco_rope(qp, q_bias, kp, k_bias, cos_cache, sin_cache, positions[r],
                 head_dim, num_q_heads, num_kv_heads, sub_mode, add_mode);
        lco_update_kv_cache(k_pool, v_pool, kp, vp, v_bias,
                            block_tables + (int64_t)b * table_stride, layer,
                            positions[r], num_layers, num_kv_heads, head_dim, 16);
    }
    return 0;
}

int lco_gather_kv(uint16_t *k_out, uint16_t *v_out, const uint16_t *k_pool,
                  const uint16_t *v_pool, int64_t num_blocks, int num_layers,
                  int layer, int num_kv_heads, int head_dim,
                  const int *block_tables, int table_stride,
                  const int *context_lens, int len_offset, int batch,
                  int max_context_len) {
    int err = 0;
    for (int b = 0; b < batch; ++b) {
        int n = context_lens[b] + len_offset;
        if (n > max_context_len) n = max_context_len;
        for (int t = 0; t < n; ++t) {
            int phys = block_tables[(int64_t)b * table_stride + t / 16];
            if (phys < 0 || phys >= num_blocks) { err = -1; continue; }
            for (int h = 0; h < num_kv_heads; ++h) {
                int64_t src = pool_offset(phys, layer, h, t % 16, num_layers,
                                          num_kv_heads, 16, head_dim);
                int64_t dst = (((int64_t)b * max_context_len + t) * num_kv_heads + h) * head_dim;
                memcpy(k_out + dst, k_pool + src, sizeof(uint16_t) * head_dim);
                memcpy(v_out + dst, v_pool + src, sizeof(uint16_t) * head_dim);
            }
        }
    }
    return err;
}

/* ------------------------------------------------------------- sampling --
 * Restatement of the reference's token selection (src/kernels/sampling.cu,
 * src/kernels/sampling_optimized.cu; launched by src/kernels.rs:322-490).
 * Ties are resolved as the reference's reductions resolve them: argmax_kernel
 * (1024 threads, cub block reduction, left operand kept on ties) prefers the
 * lowest thread i % 1024, then the first i of that thread; top_k_filter (256
 * threads, shfl_down tree over offsets 16..1 keeping its own value on ties,
 * for lanes and then for warps) prefers warps and lanes in bit-reversed order,
 * then the first index of the thread. */

static int bitrev5(int x) {
    int r = 0;
    for (int b = 0; b < 5; ++b) r |= ((x >> b) & 1) << (4 - b);
    return r;
}

/* argmax_kernel: index of the largest logit above -1e30 (-1 if none). */
int lco_argmax(const uint16_t *logits, int vocab) {
    int best = -1;
    float bv = -1e30f;
    for (int i = 0; i < vocab; ++i) {
        const float v = lco_bf16_to_f32(logits[i]);
        if (v > bv) {
            best = i, bv = v;
        } else if (v == bv && best >= 0 && (i % 1024) < (best % 1024)) {
            best = i;  /* an earlier thread holds an equal maximum */
        }
    }
    return best;
}

/* top_k_filter over 32 partitions [p*V/32, (p+1)*V/32): each yields its kpb
 * largest logits in order, by repeated block argmax with removal (a removed
 * or exhausted entry reads as -1e30 and is never chosen again). keys/values:
 * [32 * kpb], partition-major; an exhausted partition gives key start - 1 and
 * value -1e30. */
void lco_top_k_filter(const uint16_t *logits, int vocab, int kpb, int *keys, float *values) {
    for (int p = 0; p < 32; ++p) {
        const int start = (int)((long long)p * vocab / 32);
        const int end = (int)((long long)(p + 1) * vocab / 32);
        const int n = end - start;
        float *v = (float *)malloc(sizeof(float) * (n > 0 ? n : 1));
        for (int i = 0; i < n; ++i) v[i] = lco_bf16_to_f32(logits[start + i]);
        for (int k = 0; k < kpb; ++k) {
            int best = -1;
            float bv = -1e30f;
            for (int i = 0; i < n; ++i) {
                if (v[i] > bv) {
                    best = i, bv = v[i];
                } else if (v[i] == bv && best >= 0) {
                    const int t = i % 256, tb = best % 256;
                    const int pr = bitrev5(t / 32) * 32 + bitrev5(t % 32);
                    const int pb = bitrev5(tb / 32) * 32 + bitrev5(tb % 32);
                    if (pr < pb) best = i;  /* same value, preferred thread */
                }
            }
            if (n <= 0) continue;  /* the reference writes nothing for an empty partition */
            keys[p * kpb + k] = start + best;
            values[p * kpb + k] = bv;
            if (best >= 0) v[best] = -1e30f;
        }
        free(v);
    }
}

/* fused_top_p_sample_impl<n>: bitonic sort of the n candidates (descending,
 * the reference's compare-exchange network, so equal values keep its order),
 * softmax over them, the top-p cutoff and the draw. Sums here are in double;
 * *margin returns how far (in probability) the draw and the cutoff were from
 * a boundary, so that a caller comparing with fp32 arithmetic can skip draws
 * that rounding could move. Returns the chosen key, or -1 when no candidate
 * wins (the reference then leaves its output untouched). */
int lco_top_p_sample(const int *keys_in, const float *values_in, int n, float top_p,
                     float rand_val, double *margin) {
    int *keys = (int *)malloc(sizeof(int) * n);
    float *vals = (float *)malloc(sizeof(float) * n);
    memcpy(keys, keys_in, sizeof(int) * n);
    memcpy(vals, values_in, sizeof(float) * n);
    for (int k = 2; k <= n; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1)
            for (int t = 0; t < n; ++t) {
                const int o = t ^ j;
                if (o <= t) continue;
                const int sw = (t & k) == 0 ? vals[t] < vals[o] : vals[t] > vals[o];
                if (sw) {
                    const float tv = vals[t];
                    const int tk = keys[t];
                    vals[t] = vals[o], keys[t] = keys[o];
                    vals[o] = tv, keys[o] = tk;
                }
            }
    double *e = (double *)malloc(sizeof(double) * n);
    double total = 0.0;
    for (int t = 0; t < n; ++t) {
        e[t] = exp((double)vals[t] - (double)vals[0]);
        total += e[t];
    }
    double cdf = 0.0, cutoff = 1.0, m = 1.0;
    for (int t = 0; t < n; ++t) {
        const double prev = cdf;
        cdf += e[t] / total;
        if (prev < top_p && cdf >= top_p) cutoff = cdf;
        /* a cumulative value next to top_p can move the cutoff to the next
         * candidate's; past the last one the alternative is 1.0, which the
         * last cumulative value equals up to rounding */
        const double d = fabs(cdf - top_p);
        if (t < n - 1 && d < m) m = d;
    }
    const double target = (double)rand_val * cutoff;
    int chosen = -1;
    cdf = 0.0;
    for (int t = 0; t < n; ++t) {
        const double prev = cdf;
        cdf += e[t] / total;
        if (cdf >= target && prev < target) chosen = keys[t];
        const double d = fabs(cdf - target);
        if (d < m) m = d;
    }
    if (margin) *margin = m;
    free(e);
    free(keys);
    free(vals);
    return chosen;
}
