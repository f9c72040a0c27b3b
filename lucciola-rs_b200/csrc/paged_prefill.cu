// paged_prefill.cu - causal prefill over the paged KV pool (placeholder until
// the tcgen05 kernel lands: reports LC_ERR_NOT_SUPPORTED).
#include "lc_common.cuh"
#include "lc_host.h"

extern "C" int lc_paged_prefill(void *out, int64_t out_stride, const void *q, int64_t q_stride,
                                const void *k_pool, const void *v_pool, int64_t num_blocks,
                                int num_layers, int layer, int num_q_heads, int num_kv_heads,
                                int head_dim, const int *block_tables, int table_stride,
                                const int *start_pos, int num_seqs, int tokens_per_seq,
                                int max_start_pos, float sm_scale, int *dev_status,
                                lc_stream_t stream) {
    (void)out; (void)out_stride; (void)q; (void)q_stride; (void)k_pool; (void)v_pool;
    (void)num_blocks; (void)num_layers; (void)layer; (void)num_q_heads; (void)num_kv_heads;
    (void)head_dim; (void)block_tables; (void)table_stride; (void)start_pos; (void)num_seqs;
    (void)tokens_per_seq; (void)max_start_pos; (void)sm_scale; (void)dev_status; (void)stream;
    return LC_ERR_NOT_SUPPORTED;
}
