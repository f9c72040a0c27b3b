// lc_host.h - host-side helpers shared by the C-ABI implementation files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lucciola_attn.h"

namespace lc {

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline cudaStream_t as_stream(lc_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Returns LC_OK or LC_ERR_CUDA for the last launch on this thread.
inline int launch_status() {
    return cudaGetLastError() == cudaSuccess ? LC_OK : LC_ERR_CUDA;
}

// Tiled 2-D tensor map over a paged pool viewed as [rows][head_dim] bf16 with
// a {64, 16} box (one 128-byte-wide half page) and 128-byte swizzle. Maps are
// cached by (pointer, rows, head_dim); the cache is thread-safe.
// Returns LC_OK, LC_ERR_INVALID_ARGUMENT (rows beyond the int32 coordinate
// range), LC_ERR_MISALIGNED or LC_ERR_CUDA.
int pool_tensor_map(const void *pool, int64_t rows, int head_dim, CUtensorMap *out);

// The same map encoded without the cache (no host allocation).
int pool_tensor_map_nocache(const void *pool, int64_t rows, int head_dim, CUtensorMap *out);

// 2-D bf16 tensor map [rows][inner] with row pitch `row_bytes`, box
// {box_inner, box_rows}, 128-byte swizzle, zero fill out of bounds (uncached).
int tensor_map_2d_sw128(const void *base, int64_t inner, int64_t rows, int64_t row_bytes,
                        int box_inner, int box_rows, CUtensorMap *out);

// The same with a swizzle span of 0 (none), 32, 64 or 128 bytes.
int tensor_map_2d(const void *base, int64_t inner, int64_t rows, int64_t row_bytes, int box_inner,
                  int box_rows, int swizzle_bytes, CUtensorMap *out);

// Applies cudaFuncAttributeMaxDynamicSharedMemorySize once per (function, device).
int ensure_smem_attr(const void *func, int bytes);

// Number of SMs of the current device (cached per device).
int sm_count();

// Process-wide programmatic-dependent-launch mode (lc_set_dependent_launch).
int dependent_launch_mode();

// The decode-step projection (proj_decode.cu): out[M][N] = x[M][K] . w[N][K]^T
// for M <= kDecodeProjMaxRows token rows, with epilogue `epi` (0 plain,
// 1 residual, 2 QKV with bias + RoPE + paged append: the fields after
// res_stride then apply). Shapes and pointers are checked by the caller.
constexpr int kDecodeProjMaxRows = 128;
struct DecodeProjArgs {
    int epi, M, N, K;
    void *out;
    int64_t out_stride;
    const void *x;
    int64_t x_stride;
    const void *w;
    int64_t w_stride;
    const void *residual;
    int64_t res_stride;
    int tokens_per_seq;
    const int *positions;
    const void *q_bias, *k_bias, *v_bias;
    const float *cos_t, *sin_t;
    int rope_rows;
    void *k_pool, *v_pool;
    int64_t num_blocks;
    int num_layers, layer, num_q_heads, num_kv_heads, head_dim;
    const int *tables;
    int table_stride;
    int *status;
};
int decode_proj_launch(const DecodeProjArgs &a, cudaStream_t stream);

}  // namespace lc

// Peer exchange group (lc_peer_group_*): the ranks' exchange regions as this
// process addresses them. Signal words at the head of every region (int32):
// [0, 8) rank r's launch count, written by rank r into every peer's region;
// kPeerDoneWord: CTAs of the running peer decode that have finished (local);
// kPeerSeqWord: peer decode launches so far (local); kPeerWaitWord: waits so
// far (local).
struct lc_peer_group {
    int rank, world;
    size_t bytes;
    uint8_t *region[LC_PEER_MAX_RANKS];
    bool opened[LC_PEER_MAX_RANKS];  // mapped by lc_peer_group_open (closed on destroy)
};

namespace lc {
constexpr int kPeerDoneWord = 16, kPeerSeqWord = 17, kPeerWaitWord = 18;
static_assert((kPeerWaitWord + 1) * 4 <= LC_PEER_SIGNAL_BYTES, "signal words fit");
}  // namespace lc
