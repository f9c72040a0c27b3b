// layers.cpp - host-side mirror of the reference's Rust layer objects on the
// attention path: RopeCache (src/layers/rope.rs), KVCache
// (src/layers/kv_cache.rs) and CudaFunctions::apply_flash_decoding
// (src/kernels.rs:248-320). These own device memory, as the reference's cudarc
// slices do; the kernels they launch are the C-ABI entry points.
#include <cmath>
#include <new>
#include <vector>

#include "../lc_host.h"

// ------------------------------------------------------------- RopeCache --

extern "C" void lc_rope_table_host(int max_position_embeddings, int head_dim, float base,
                                   float scale_factor, float *cos_out, float *sin_out) {
    // src/layers/rope.rs:21-31, f32 throughout: t = pos / scale,
    // theta = t / base.powf((2i) / hd), then cos/sin.
    const int half = head_dim / 2;
    const float scale = scale_factor > 0.0f ? scale_factor : 1.0f;
    for (int pos = 0; pos < max_position_embeddings; ++pos) {
        for (int i = 0; i < half; ++i) {
            const float t = static_cast<float>(pos) / scale;
            const float theta =
                t / std::pow(base, static_cast<float>(2 * i) / static_cast<float>(head_dim));
            cos_out[(int64_t)pos * half + i] = std::cos(theta);
            sin_out[(int64_t)pos * half + i] = std::sin(theta);
        }
    }
}

struct lc_rope_cache {
    float *cos = nullptr;
    float *sin = nullptr;
};

extern "C" int lc_rope_cache_new(int max_position_embeddings, int head_dim, float base,
                                 float scale_factor, lc_stream_t stream, lc_rope_cache **out) {
    if (!out || max_position_embeddings <= 0 || head_dim <= 0 || (head_dim & 1))
        return LC_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    const size_t n = (size_t)max_position_embeddings * (head_dim / 2);
    std::vector<float> c(n), s(n);
    lc_rope_table_host(max_position_embeddings, head_dim, base, scale_factor, c.data(), s.data());
    auto *rc = new (std::nothrow) lc_rope_cache();
    if (!rc) return LC_ERR_OUT_OF_MEMORY;
    cudaStream_t st = lc::as_stream(stream);
    if (cudaMalloc(&rc->cos, n * 4) != cudaSuccess || cudaMalloc(&rc->sin, n * 4) != cudaSuccess ||
        cudaMemcpyAsync(rc->cos, c.data(), n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(rc->sin, s.data(), n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        lc_rope_cache_free(rc);
        return LC_ERR_CUDA;
    }
    *out = rc;
    return LC_OK;
}

extern "C" const float *lc_rope_cache_cos(const lc_rope_cache *rc) { return rc ? rc->cos : nullptr; }
extern "C" const float *lc_rope_cache_sin(const lc_rope_cache *rc) { return rc ? rc->sin : nullptr; }

extern "C" void lc_rope_cache_free(lc_rope_cache *rc) {
    if (!rc) return;
    cudaFree(rc->cos);
    cudaFree(rc->sin);
    delete rc;
}

// --------------------------------------------------------------- KVCache --

struct lc_kv_cache {
    void *k_pool = nullptr;
    void *v_pool = nullptr;
    int *block_table = nullptr;
    std::vector<int> block_table_cpu;
    std::vector<int> free_blocks;
    int block_size = 16;
    int64_t num_physical_blocks = 0;
    int max_seq_len = 0;
    int max_logical_blocks = 0;
    int num_q_heads = 0;
    int num_kv_heads = 0;
    int head_dim = 0;
    int num_layers = 0;
    void *workspace = nullptr;  // split-K scratch for lc_apply_flash_decoding
    size_t workspace_bytes = 0;
};

extern "C" void lc_kv_cache_free(lc_kv_cache *c) {
    if (!c) return;
    cudaFree(c->k_pool);
    cudaFree(c->v_pool);
    cudaFree(c->block_table);
    cudaFree(c->workspace);
    delete c;
}

extern "C" int lc_kv_cache_new(int num_hidden_layers, int num_attention_heads,
                               int num_key_value_heads, int head_dim,
                               int max_position_embeddings, float memory_fraction,
                               lc_stream_t stream, lc_kv_cache **out) {
    if (!out || num_hidden_layers <= 0 || num_attention_heads <= 0 || num_key_value_heads <= 0 ||
        head_dim <= 0 || max_position_embeddings <= 0 || !(memory_fraction > 0.0f))
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (num_attention_heads % num_key_value_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    *out = nullptr;
    const int block_size = 16;
    // kv_cache.rs:37-48: budget = total * fraction (in f32) - used.
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return LC_ERR_CUDA;
    const size_t used = total_b - free_b;
    const size_t available_total = (size_t)((float)total_b * memory_fraction);
    if (available_total < used) return LC_ERR_OUT_OF_MEMORY;
    const size_t allocatable = available_total - used;
    // kv_cache.rs:50-59
    const size_t bytes_per_block =
        2ull * num_hidden_layers * num_key_value_heads * block_size * head_dim * 2;
    const int max_logical = (max_position_embeddings + block_size - 1) / block_size;
    size_t blocks = allocatable / bytes_per_block;
    if (blocks > (size_t)max_logical) blocks = max_logical;
    const size_t pool_elems = blocks * num_hidden_layers * num_key_value_heads * block_size * head_dim;

    auto *c = new (std::nothrow) lc_kv_cache();
    if (!c) return LC_ERR_OUT_OF_MEMORY;
    c->num_physical_blocks = (int64_t)blocks;
    c->max_seq_len = max_position_embeddings;
    c->max_logical_blocks = max_logical;
    c->num_q_heads = num_attention_heads;
    c->num_kv_heads = num_key_value_heads;
    c->head_dim = head_dim;
    c->num_layers = num_hidden_layers;
    c->workspace_bytes =
        lc_flash_decoding_workspace_size(num_attention_heads, head_dim, max_position_embeddings);
    cudaStream_t st = lc::as_stream(stream);
    const size_t pool_bytes = pool_elems * 2;
    if ((pool_bytes && cudaMalloc(&c->k_pool, pool_bytes) != cudaSuccess) ||
        (pool_bytes && cudaMalloc(&c->v_pool, pool_bytes) != cudaSuccess) ||
        cudaMalloc(&c->block_table, (size_t)max_logical * 4) != cudaSuccess ||
        cudaMalloc(&c->workspace, c->workspace_bytes) != cudaSuccess) {
        lc_kv_cache_free(c);
        return LC_ERR_OUT_OF_MEMORY;
    }
    if ((pool_bytes && (cudaMemsetAsync(c->k_pool, 0, pool_bytes, st) != cudaSuccess ||
                        cudaMemsetAsync(c->v_pool, 0, pool_bytes, st) != cudaSuccess)) ||
        cudaMemsetAsync(c->block_table, 0, (size_t)max_logical * 4, st) != cudaSuccess ||
        cudaMemsetAsync(c->workspace, 0, c->workspace_bytes, st) != cudaSuccess) {
        lc_kv_cache_free(c);
        return LC_ERR_CUDA;
    }
    // kv_cache.rs:73-76: pushed in reverse so that pops yield 0, 1, 2, ...
    c->free_blocks.reserve(blocks);
    for (int64_t i = (int64_t)blocks - 1; i >= 0; --i) c->free_blocks.push_back((int)i);
    *out = c;
    return LC_OK;
}

extern "C" int lc_kv_cache_prepare_for_step(lc_kv_cache *c, lc_stream_t stream, int pos) {
    if (!c || pos < 0) return LC_ERR_INVALID_ARGUMENT;
    const int logical = pos / c->block_size;
    if (logical >= c->max_logical_blocks) return LC_ERR_INVALID_ARGUMENT;
    if (logical < (int)c->block_table_cpu.size()) return LC_OK;
    while ((int)c->block_table_cpu.size() <= logical) {
        if (c->free_blocks.empty()) return LC_ERR_OUT_OF_BLOCKS;  // kv_cache.rs:110-113 panics
        c->block_table_cpu.push_back(c->free_blocks.back());
        c->free_blocks.pop_back();
    }
    // kv_cache.rs:116-119: the whole host table goes to the device.
    if (cudaMemcpyAsync(c->block_table, c->block_table_cpu.data(), c->block_table_cpu.size() * 4,
                        cudaMemcpyHostToDevice, lc::as_stream(stream)) != cudaSuccess)
        return LC_ERR_CUDA;
    return LC_OK;
}

extern "C" int lc_kv_cache_update(lc_kv_cache *c, lc_stream_t stream, int layer_idx, int pos,
                                  const int *pos_ptr, const void *k_input, const void *v_input,
                                  const void *v_bias) {
    if (!c) return LC_ERR_INVALID_ARGUMENT;
    int rc = lc_kv_cache_prepare_for_step(c, stream, pos);
    if (rc) return rc;
    return lc_update_kv_cache(c->k_pool, c->v_pool, k_input, v_input, v_bias, c->block_table,
                              layer_idx, pos_ptr, c->num_layers, c->num_kv_heads, c->max_seq_len,
                              c->head_dim, c->block_size, stream);
}

extern "C" void *lc_kv_cache_k_pool(lc_kv_cache *c) { return c ? c->k_pool : nullptr; }
extern "C" void *lc_kv_cache_v_pool(lc_kv_cache *c) { return c ? c->v_pool : nullptr; }
extern "C" int *lc_kv_cache_block_table(lc_kv_cache *c) { return c ? c->block_table : nullptr; }
extern "C" int64_t lc_kv_cache_num_physical_blocks(const lc_kv_cache *c) {
    return c ? c->num_physical_blocks : 0;
}
extern "C" int lc_kv_cache_max_seq_len(const lc_kv_cache *c) { return c ? c->max_seq_len : 0; }
extern "C" int lc_kv_cache_num_allocated_blocks(const lc_kv_cache *c) {
    return c ? (int)c->block_table_cpu.size() : 0;
}

extern "C" int lc_apply_flash_decoding(lc_kv_cache *c, lc_stream_t stream, void *output,
                                       const void *q, int layer_idx, int pos, const int *pos_ptr,
                                       int num_q_heads) {
    if (!c) return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads != c->num_q_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    const float scale = 1.0f / std::sqrt((float)c->head_dim);  // kernels.rs:264
    return lc_flash_decoding(output, q, c->k_pool, c->v_pool, c->block_table, layer_idx,
                             num_q_heads, c->num_kv_heads, c->head_dim, c->max_seq_len, pos_ptr,
                             scale, c->block_size, c->num_layers, pos, c->num_physical_blocks,
                             c->workspace, c->workspace_bytes, stream);
}
