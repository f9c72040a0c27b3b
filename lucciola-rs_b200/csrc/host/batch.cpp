// batch.cpp - the batched token-step driver around the attention path: a
// paged KV pool shared by many sequences (one block-table row per sequence,
// one LIFO free list of 16-token pages) and the per-step / per-layer calls that
// run a batched decode or a prompt prefill on it.
//
// The reference keeps one KVCache per model, i.e. one sequence
// (src/layers/kv_cache.rs:12-174: a single block table, prepare_for_step pushes
// the next block and copies the whole table to the device, :106-122), and its
// decode loop runs one token of one sequence per step (src/models.rs:230-245,
// attention section :486-550). Here:
//   * lc_block_alloc holds the page bookkeeping only (host memory): slots for
//     sequences, their page lists, the free list. Pages come out 0, 1, 2, ...
//     from a fresh pool as in kv_cache.rs:73-76; a released sequence's pages go
//     back so that the next sequence gets them in the same order.
//   * lc_kv_pool owns the device side: the K and V pools
//     [num_blocks][num_layers][num_kv_heads][16][head_dim] bf16, the step's
//     block tables in batch order and the new tokens' positions (device
//     buffers at fixed addresses, so that the per-layer launches can be
//     captured once in a CUDA graph and replayed every step), and the split-K
//     workspace of lc_rope_append_decode.
//   * lc_kv_pool_prepare_step reserves the pages each sequence of the step
//     needs and uploads the step's tables and positions (one copy each from
//     pinned staging, double-buffered so that the host never waits for the copy
//     it just issued); lc_kv_pool_decode_layer is then one lc_rope_append_decode
//     launch per layer.
#include <algorithm>
#include <climits>
#include <cmath>
#include <new>
#include <vector>

#include "../lc_host.h"

namespace {
constexpr int kBlockSize = 16;  // tokens per page (src/layers/kv_cache.rs:35)
}

// --------------------------------------------------------- page bookkeeping --

struct lc_block_alloc {
    int64_t num_blocks = 0;
    int max_seqs = 0;
    int max_blocks_per_seq = 0;
    std::vector<int> free_list;           // LIFO: back() is handed out next
    std::vector<std::vector<int>> pages;  // per slot, logical page -> physical page
    std::vector<char> live;               // slot in use
};

extern "C" int lc_block_alloc_new(int64_t num_blocks, int max_seqs, int max_blocks_per_seq,
                                  lc_block_alloc **out) {
    if (!out || num_blocks <= 0 || num_blocks > INT32_MAX || max_seqs <= 0 ||
        max_blocks_per_seq <= 0)
        return LC_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    auto *a = new (std::nothrow) lc_block_alloc();
    if (!a) return LC_ERR_OUT_OF_MEMORY;
    try {
        a->num_blocks = num_blocks;
        a->max_seqs = max_seqs;
        a->max_blocks_per_seq = max_blocks_per_seq;
        a->free_list.reserve((size_t)num_blocks);
        for (int64_t i = num_blocks - 1; i >= 0; --i) a->free_list.push_back((int)i);
        a->pages.resize((size_t)max_seqs);
        a->live.assign((size_t)max_seqs, 0);
    } catch (...) {
        delete a;
        return LC_ERR_OUT_OF_MEMORY;
    }
    *out = a;
    return LC_OK;
}

extern "C" void lc_block_alloc_free(lc_block_alloc *a) { delete a; }

extern "C" int lc_block_alloc_add_seq(lc_block_alloc *a, int *slot) {
    if (!a || !slot) return LC_ERR_INVALID_ARGUMENT;
    for (int s = 0; s < a->max_seqs; ++s)
        if (!a->live[s]) {
            a->live[s] = 1;
            a->pages[s].clear();
            *slot = s;
            return LC_OK;
        }
    return LC_ERR_NO_FREE_SLOT;
}

static bool slot_ok(const lc_block_alloc *a, int slot) {
    return a && slot >= 0 && slot < a->max_seqs && a->live[slot];
}

extern "C" int lc_block_alloc_release_seq(lc_block_alloc *a, int slot) {
    if (!slot_ok(a, slot)) return LC_ERR_INVALID_ARGUMENT;
    std::vector<int> &pg = a->pages[slot];
    // Last page first, so that the free list hands them out again in order.
    for (auto it = pg.rbegin(); it != pg.rend(); ++it) a->free_list.push_back(*it);
    pg.clear();
    a->live[slot] = 0;
    return LC_OK;
}

extern "C" int lc_block_alloc_reserve(lc_block_alloc *a, int slot, int tokens) {
    if (!slot_ok(a, slot) || tokens < 0) return LC_ERR_INVALID_ARGUMENT;
    const int need = (tokens + kBlockSize - 1) / kBlockSize;
    if (need > a->max_blocks_per_seq) return LC_ERR_INVALID_ARGUMENT;  // beyond the table row
    std::vector<int> &pg = a->pages[slot];
    if ((int)pg.size() >= need) return LC_OK;
    if ((int64_t)(need - pg.size()) > (int64_t)a->free_list.size()) return LC_ERR_OUT_OF_BLOCKS;
    while ((int)pg.size() < need) {
        pg.push_back(a->free_list.back());
        a->free_list.pop_back();
    }
    return LC_OK;
}

extern "C" int lc_block_alloc_row(const lc_block_alloc *a, int slot, int *dst, int capacity) {
    if (!slot_ok(a, slot) || (!dst && capacity > 0) || capacity < 0) return -1;
    const std::vector<int> &pg = a->pages[slot];
    const int n = std::min<int>((int)pg.size(), capacity);
    std::copy(pg.begin(), pg.begin() + n, dst);
    return (int)pg.size();
}

extern "C" int64_t lc_block_alloc_num_free(const lc_block_alloc *a) {
    return a ? (int64_t)a->free_list.size() : 0;
}

extern "C" uint64_t lc_block_alloc_fingerprint(const lc_block_alloc *a) {
    if (!a) return 0;
    // FNV-1a over everything that decides future tables: each slot's state and
    // pages, then the free list in hand-out order.
    uint64_t h = 1469598103934665603ull;
    auto mix = [&h](int64_t v) {
        for (int i = 0; i < 8; ++i) {
            h ^= (uint64_t)((v >> (8 * i)) & 0xff);
            h *= 1099511628211ull;
        }
    };
    mix(a->num_blocks);
    mix(a->max_seqs);
    mix(a->max_blocks_per_seq);
    for (int s = 0; s < a->max_seqs; ++s) {
        mix(a->live[s]);
        mix((int64_t)a->pages[s].size());
        for (int pg : a->pages[s]) mix(pg);
    }
    mix((int64_t)a->free_list.size());
    for (int pg : a->free_list) mix(pg);
    return h;
}

// ------------------------------------------------------------- pool sizing --

extern "C" int64_t lc_kv_pool_blocks_for_budget(int num_layers, int num_kv_heads, int head_dim,
                                                uint64_t free_bytes, uint64_t total_bytes,
                                                float memory_fraction) {
    if (num_layers <= 0 || num_kv_heads <= 0 || head_dim <= 0 || !(memory_fraction > 0.0f) ||
        free_bytes > total_bytes)
        return 0;
    // src/layers/kv_cache.rs:37-59: budget = total * fraction (in f32) - used,
    // divided by the K+V bytes of one 16-token page over all layers. No cap at
    // one sequence's pages: the pool is shared by many sequences.
    const uint64_t used = total_bytes - free_bytes;
    const uint64_t available_total = (uint64_t)((float)total_bytes * memory_fraction);
    if (available_total <= used) return 0;
    const uint64_t bytes_per_block =
        2ull * num_layers * num_kv_heads * kBlockSize * (uint64_t)head_dim * 2;
    int64_t blocks = (int64_t)((available_total - used) / bytes_per_block);
    // pool rows (blocks x layers x heads x 16) must fit the kernels' int32 row index
    const int64_t row_cap = ((int64_t(1) << 31) - 1) / ((int64_t)num_layers * num_kv_heads * kBlockSize);
    return std::min(blocks, row_cap);
}

extern "C" int lc_kv_pool_capacity(int num_layers, int num_kv_heads, int head_dim,
                                   float memory_fraction, int64_t *num_blocks) {
    if (!num_blocks) return LC_ERR_INVALID_ARGUMENT;
    *num_blocks = 0;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    *num_blocks = lc_kv_pool_blocks_for_budget(num_layers, num_kv_heads, head_dim, free_b,
                                               total_b, memory_fraction);
    return *num_blocks > 0 ? LC_OK : LC_ERR_OUT_OF_MEMORY;
}

// -------------------------------------------------------------- device pool --

struct lc_kv_pool {
    lc_block_alloc *alloc = nullptr;
    int num_layers = 0, num_q_heads = 0, num_kv_heads = 0, head_dim = 0;
    int max_seqs = 0, max_blocks = 0;
    int64_t num_blocks = 0;
    void *k_pool = nullptr, *v_pool = nullptr;
    int *d_tables = nullptr;     // [max_seqs][max_blocks]: the step's rows, batch order
    int *d_positions = nullptr;  // [max_seqs]: the step's new-token positions
    int *h_stage[2] = {nullptr, nullptr};  // pinned: tables then positions
    cudaEvent_t stage_done[2] = {nullptr, nullptr};
    int stage = 0;
    int batch = 0;
    // prompt prefill of one sequence
    int *d_pf_table = nullptr;   // [max_blocks]
    int *d_pf_pos = nullptr;     // [max_blocks * 16]: positions of the prompt rows
    int *d_pf_start = nullptr;   // [1]
    int pf_tokens = 0, pf_start = 0;
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
};

extern "C" void lc_kv_pool_free(lc_kv_pool *p) {
    if (!p) return;
    for (int i = 0; i < 2; ++i) {
        if (p->stage_done[i]) {
            cudaEventSynchronize(p->stage_done[i]);
            cudaEventDestroy(p->stage_done[i]);
        }
        cudaFreeHost(p->h_stage[i]);
    }
    cudaFree(p->k_pool);
    cudaFree(p->v_pool);
    cudaFree(p->d_tables);
    cudaFree(p->d_positions);
    cudaFree(p->d_pf_table);
    cudaFree(p->d_pf_pos);
    cudaFree(p->d_pf_start);
    cudaFree(p->workspace);
    lc_block_alloc_free(p->alloc);
    delete p;
}

static size_t stage_ints(const lc_kv_pool *p) {
    // decode: tables + positions; prefill: one table row + positions + start
    const size_t dec = (size_t)p->max_seqs * p->max_blocks + p->max_seqs;
    const size_t pf = (size_t)p->max_blocks + (size_t)p->max_blocks * kBlockSize + 1;
    return std::max(dec, pf);
}

extern "C" int lc_kv_pool_new(int num_layers, int num_q_heads, int num_kv_heads, int head_dim,
                              int max_seqs, int max_seq_len, int64_t num_blocks,
                              lc_stream_t stream, lc_kv_pool **out) {
    if (!out || num_layers <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_seqs <= 0 ||
        max_seq_len <= 0 || num_blocks <= 0)
        return LC_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return LC_ERR_UNSUPPORTED_HEAD_DIM;
    if (num_q_heads % num_kv_heads) return LC_ERR_UNSUPPORTED_SHAPE;
    if (num_blocks * num_layers * num_kv_heads * kBlockSize >= (int64_t(1) << 31))
        return LC_ERR_INVALID_ARGUMENT;  // pool rows must fit the kernels' int32 row index
    *out = nullptr;
    auto *p = new (std::nothrow) lc_kv_pool();
    if (!p) return LC_ERR_OUT_OF_MEMORY;
    p->num_layers = num_layers;
    p->num_q_heads = num_q_heads;
    p->num_kv_heads = num_kv_heads;
    p->head_dim = head_dim;
    p->max_seqs = max_seqs;
    p->max_blocks = (max_seq_len + kBlockSize - 1) / kBlockSize;
    p->num_blocks = num_blocks;
    int rc = lc_block_alloc_new(num_blocks, max_seqs, p->max_blocks, &p->alloc);
    if (rc) {
        lc_kv_pool_free(p);
        return rc;
    }
    const size_t pool_bytes =
        (size_t)num_blocks * num_layers * num_kv_heads * kBlockSize * head_dim * 2;
    p->workspace_bytes = lc_paged_decode_workspace_size(max_seqs, num_q_heads, num_kv_heads, head_dim);
    const size_t sint = stage_ints(p);
    cudaStream_t st = lc::as_stream(stream);
    if (cudaMalloc(&p->k_pool, pool_bytes) != cudaSuccess ||
        cudaMalloc(&p->v_pool, pool_bytes) != cudaSuccess ||
        cudaMalloc(&p->d_tables, (size_t)max_seqs * p->max_blocks * 4) != cudaSuccess ||
        cudaMalloc(&p->d_positions, (size_t)max_seqs * 4) != cudaSuccess ||
        cudaMalloc(&p->d_pf_table, (size_t)p->max_blocks * 4) != cudaSuccess ||
        cudaMalloc(&p->d_pf_pos, (size_t)p->max_blocks * kBlockSize * 4) != cudaSuccess ||
        cudaMalloc(&p->d_pf_start, 4) != cudaSuccess ||
        cudaMalloc(&p->workspace, p->workspace_bytes) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void **>(&p->h_stage[0]), sint * 4, cudaHostAllocDefault) !=
            cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void **>(&p->h_stage[1]), sint * 4, cudaHostAllocDefault) !=
            cudaSuccess ||
        cudaEventCreateWithFlags(&p->stage_done[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&p->stage_done[1], cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        lc_kv_pool_free(p);
        return LC_ERR_OUT_OF_MEMORY;
    }
    if (cudaMemsetAsync(p->k_pool, 0, pool_bytes, st) != cudaSuccess ||
        cudaMemsetAsync(p->v_pool, 0, pool_bytes, st) != cudaSuccess ||
        cudaMemsetAsync(p->d_tables, 0, (size_t)max_seqs * p->max_blocks * 4, st) != cudaSuccess ||
        cudaMemsetAsync(p->d_positions, 0, (size_t)max_seqs * 4, st) != cudaSuccess ||
        lc_paged_decode_workspace_init(p->workspace, p->workspace_bytes, stream) != LC_OK ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        cudaGetLastError();
        lc_kv_pool_free(p);
        return LC_ERR_CUDA;
    }
    *out = p;
    return LC_OK;
}

extern "C" int lc_kv_pool_add_sequence(lc_kv_pool *p, int *slot) {
    return p ? lc_block_alloc_add_seq(p->alloc, slot) : LC_ERR_INVALID_ARGUMENT;
}

extern "C" int lc_kv_pool_release_sequence(lc_kv_pool *p, int slot) {
    return p ? lc_block_alloc_release_seq(p->alloc, slot) : LC_ERR_INVALID_ARGUMENT;
}

// Next pinned staging buffer, after the copy that last read it has finished.
static int take_stage(lc_kv_pool *p, int **buf) {
    p->stage ^= 1;
    if (cudaEventSynchronize(p->stage_done[p->stage]) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    *buf = p->h_stage[p->stage];
    return LC_OK;
}

extern "C" int lc_kv_pool_prepare_step(lc_kv_pool *p, lc_stream_t stream, int batch,
                                       const int *slots, const int *positions) {
    if (!p || batch <= 0 || batch > p->max_seqs || !slots || !positions)
        return LC_ERR_INVALID_ARGUMENT;
    for (int b = 0; b < batch; ++b) {
        if (positions[b] < 0) return LC_ERR_INVALID_ARGUMENT;
        for (int c = 0; c < b; ++c)
            if (slots[c] == slots[b]) return LC_ERR_INVALID_ARGUMENT;  // one row per sequence
        // The new token at positions[b] needs positions[b] + 1 cached tokens.
        const int rc = lc_block_alloc_reserve(p->alloc, slots[b], positions[b] + 1);
        if (rc) return rc;
    }
    int *h = nullptr;
    int rc = take_stage(p, &h);
    if (rc) return rc;
    int *tab = h, *pos = h + (size_t)batch * p->max_blocks;
    for (int b = 0; b < batch; ++b) {
        int *row = tab + (size_t)b * p->max_blocks;
        const int n = lc_block_alloc_row(p->alloc, slots[b], row, p->max_blocks);
        std::fill(row + n, row + p->max_blocks, 0);
        pos[b] = positions[b];
    }
    cudaStream_t st = lc::as_stream(stream);
    if (cudaMemcpyAsync(p->d_tables, tab, (size_t)batch * p->max_blocks * 4,
                        cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(p->d_positions, pos, (size_t)batch * 4, cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaEventRecord(p->stage_done[p->stage], st) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    p->batch = batch;
    return LC_OK;
}

extern "C" int lc_kv_pool_decode_layer(lc_kv_pool *p, lc_stream_t stream, int layer, void *out,
                                       int64_t out_stride, const void *qkv, int64_t row_stride,
                                       const void *q_bias, const void *k_bias, const void *v_bias,
                                       const float *cos_cache, const float *sin_cache,
                                       int rope_rows, int *dev_status) {
    if (!p || p->batch <= 0) return LC_ERR_INVALID_ARGUMENT;
    // No context hint: the grid is sized on the device from the positions, so
    // a captured launch stays valid as the sequences grow.
    return lc_rope_append_decode(out, out_stride, qkv, row_stride, p->d_positions, q_bias, k_bias,
                                 v_bias, cos_cache, sin_cache, rope_rows, p->k_pool, p->v_pool,
                                 p->num_blocks, p->num_layers, layer, p->num_q_heads,
                                 p->num_kv_heads, p->head_dim, p->d_tables, p->max_blocks,
                                 p->batch, 0, 0, 1.0f / std::sqrt((float)p->head_dim),
                                 p->workspace, p->workspace_bytes, dev_status, stream);
}

extern "C" int lc_kv_pool_prepare_prefill(lc_kv_pool *p, lc_stream_t stream, int slot,
                                          int start_pos, int tokens) {
    if (!p || start_pos < 0 || tokens <= 0) return LC_ERR_INVALID_ARGUMENT;
    int rc = lc_block_alloc_reserve(p->alloc, slot, start_pos + tokens);
    if (rc) return rc;
    int *h = nullptr;
    rc = take_stage(p, &h);
    if (rc) return rc;
    int *row = h, *pos = h + p->max_blocks, *st0 = pos + (size_t)p->max_blocks * kBlockSize;
    const int n = lc_block_alloc_row(p->alloc, slot, row, p->max_blocks);
    std::fill(row + n, row + p->max_blocks, 0);
    for (int i = 0; i < tokens; ++i) pos[i] = start_pos + i;
    *st0 = start_pos;
    cudaStream_t st = lc::as_stream(stream);
    if (cudaMemcpyAsync(p->d_pf_table, row, (size_t)p->max_blocks * 4, cudaMemcpyHostToDevice,
                        st) != cudaSuccess ||
        cudaMemcpyAsync(p->d_pf_pos, pos, (size_t)tokens * 4, cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaMemcpyAsync(p->d_pf_start, st0, 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaEventRecord(p->stage_done[p->stage], st) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    p->pf_tokens = tokens;
    p->pf_start = start_pos;
    return LC_OK;
}

extern "C" int lc_kv_pool_prefill_layer(lc_kv_pool *p, lc_stream_t stream, int layer, void *out,
                                        int64_t out_stride, void *qkv, int64_t row_stride,
                                        const void *q_bias, const void *k_bias, const void *v_bias,
                                        const float *cos_cache, const float *sin_cache,
                                        int rope_rows, int *dev_status) {
    if (!p || p->pf_tokens <= 0) return LC_ERR_INVALID_ARGUMENT;
    int rc = lc_rope_append(qkv, row_stride, 1, p->pf_tokens, p->d_pf_pos, q_bias, k_bias, v_bias,
                            cos_cache, sin_cache, rope_rows, p->k_pool, p->v_pool, p->num_blocks,
                            p->num_layers, layer, p->num_q_heads, p->num_kv_heads, p->head_dim,
                            p->d_pf_table, p->max_blocks, dev_status, stream);
    if (rc) return rc;
    return lc_paged_prefill(out, out_stride, qkv, row_stride, p->k_pool, p->v_pool, p->num_blocks,
                            p->num_layers, layer, p->num_q_heads, p->num_kv_heads, p->head_dim,
                            p->d_pf_table, p->max_blocks, p->d_pf_start, 1, p->pf_tokens,
                            p->pf_start, 1.0f / std::sqrt((float)p->head_dim), dev_status, stream);
}

extern "C" int lc_kv_pool_recover(lc_kv_pool *p, lc_stream_t stream) {
    if (!p) return LC_ERR_INVALID_ARGUMENT;
    return lc_paged_decode_workspace_init(p->workspace, p->workspace_bytes, stream);
}

extern "C" uint64_t lc_kv_pool_fingerprint(const lc_kv_pool *p) {
    return p ? lc_block_alloc_fingerprint(p->alloc) : 0;
}

extern "C" void *lc_kv_pool_k_pool(lc_kv_pool *p) { return p ? p->k_pool : nullptr; }
extern "C" void *lc_kv_pool_v_pool(lc_kv_pool *p) { return p ? p->v_pool : nullptr; }
extern "C" const int *lc_kv_pool_step_tables(const lc_kv_pool *p) {
    return p ? p->d_tables : nullptr;
}
extern "C" const int *lc_kv_pool_step_positions(const lc_kv_pool *p) {
    return p ? p->d_positions : nullptr;
}
extern "C" int lc_kv_pool_table_stride(const lc_kv_pool *p) { return p ? p->max_blocks : 0; }
extern "C" int64_t lc_kv_pool_num_blocks(const lc_kv_pool *p) { return p ? p->num_blocks : 0; }
extern "C" int64_t lc_kv_pool_num_free_blocks(const lc_kv_pool *p) {
    return p ? lc_block_alloc_num_free(p->alloc) : 0;
}
extern "C" int lc_kv_pool_sequence_pages(const lc_kv_pool *p, int slot, int *dst, int capacity) {
    return p ? lc_block_alloc_row(p->alloc, slot, dst, capacity) : -1;
}
