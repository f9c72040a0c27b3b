// gather.cu - dense copy of paged K/V through per-sequence block tables.
//
// Uses the same page addressing as the attention kernels (page_row), so the
// bit-exactness of this copy against the CPU oracle pins the block-table
// gather of the hot path. One CTA per (page, kv head, sequence); 16-byte loads.
#include "lc_common.cuh"
#include "lc_host.h"

namespace lc {
namespace {

struct GatherParams {
    bf16 *k_out, *v_out;
    const bf16 *k_pool, *v_pool;
    int64_t num_blocks;
    int num_layers, layer, num_kv_heads, head_dim;
    const int *tables;
    int table_stride;
    const int *ctx_lens;
    int len_offset, max_ctx;
    int *status;
};

__global__ void __launch_bounds__(128) gather_kv_kernel(GatherParams p) {
    const int page = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    int n = p.ctx_lens[b] + p.len_offset;
    if (n > p.max_ctx) n = p.max_ctx;
    if (n > p.table_stride * kBlockSize) n = p.table_stride * kBlockSize;
    const int t0 = page * kBlockSize;
    if (t0 >= n) return;
    const int valid = min(kBlockSize, n - t0);
    const int phys = p.tables[(int64_t)b * p.table_stride + page];
    if (phys < 0 || phys >= p.num_blocks) {
        if (threadIdx.x == 0) set_status(p.status, LC_DEV_BAD_BLOCK);
        return;
    }
    const int64_t src = page_row(phys, p.layer, h, p.num_layers, p.num_kv_heads) * p.head_dim;
    const int vec_per_row = p.head_dim / 8;  // 16-byte vectors
    for (int i = threadIdx.x; i < valid * vec_per_row; i += blockDim.x) {
        const int t = i / vec_per_row, v = i - t * vec_per_row;
        const int64_t dst =
            (((int64_t)b * p.max_ctx + t0 + t) * p.num_kv_heads + h) * p.head_dim + v * 8;
        const int64_t s = src + (int64_t)t * p.head_dim + v * 8;
        *reinterpret_cast<uint4 *>(p.k_out + dst) = __ldg(reinterpret_cast<const uint4 *>(p.k_pool + s));
        *reinterpret_cast<uint4 *>(p.v_out + dst) = __ldg(reinterpret_cast<const uint4 *>(p.v_pool + s));
    }
}

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" int lc_gather_kv(void *k_out, void *v_out, const void *k_pool, const void *v_pool,
                            int64_t num_blocks, int num_layers, int layer, int num_kv_heads,
                            int head_dim, const int *block_tables, int table_stride,
                            const int *context_lens, int len_offset, int batch,
                            int max_context_len, int *dev_status, lc_stream_t stream) {
    if (!k_out || !v_out || !k_pool || !v_pool || !block_tables || !context_lens)
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (batch < 0 || batch > 65535 || num_layers <= 0 || layer < 0 || layer >= num_layers ||
        num_kv_heads <= 0 || num_kv_heads > 65535 || num_blocks <= 0 || table_stride <= 0 ||
        max_context_len < 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (!aligned16(k_out) || !aligned16(v_out) || !aligned16(k_pool) || !aligned16(v_pool))
        return LC_ERR_MISALIGNED;
    if (batch == 0 || max_context_len == 0) return LC_OK;
    GatherParams p{(bf16 *)k_out, (bf16 *)v_out, (const bf16 *)k_pool, (const bf16 *)v_pool,
                   num_blocks, num_layers, layer, num_kv_heads, head_dim, block_tables,
                   table_stride, context_lens, len_offset, max_context_len, dev_status};
    dim3 grid((max_context_len + kBlockSize - 1) / kBlockSize, num_kv_heads, batch);
    gather_kv_kernel<<<grid, 128, 0, as_stream(stream)>>>(p);
    return launch_status();
}
