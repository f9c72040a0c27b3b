// ref_sampling.cu - test-side checker, never linked into the product library.
// Launches the reference's token-selection kernels, compiled unchanged from
// the reference's sources (sampling_optimized.cu), the way
// CudaFunctions::apply_sort_and_sample launches them (src/kernels.rs:346-490):
// top_k_filter on 32 blocks of 256 threads with (vocab / 32 + 256) floats of
// shared memory, then fused_top_p_sample_<n> on one block of n = 32 * (top_k /
// 32) threads.
#include <cuda_runtime.h>

#include "sampling_optimized.cu"

extern "C" int ref_sample_top_p(const void *logits, int vocab, int top_k, float top_p,
                                float rand_val, void *candidates, unsigned *out, void *stream) {
    const int grid = 32, kpb = top_k / grid, total = grid * kpb;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    KeyValuePair *cand = static_cast<KeyValuePair *>(candidates);
    top_k_filter<<<grid, 256, (size_t)((vocab / grid) + 256) * 4, s>>>(
        static_cast<const __nv_bfloat16 *>(logits), cand, vocab, kpb);
    switch (total) {
        case 32: fused_top_p_sample_32<<<1, 32, 0, s>>>(cand, top_p, rand_val, out); break;
        case 64: fused_top_p_sample_64<<<1, 64, 0, s>>>(cand, top_p, rand_val, out); break;
        case 128: fused_top_p_sample_128<<<1, 128, 0, s>>>(cand, top_p, rand_val, out); break;
        case 256: fused_top_p_sample_256<<<1, 256, 0, s>>>(cand, top_p, rand_val, out); break;
        case 512: fused_top_p_sample_512<<<1, 512, 0, s>>>(cand, top_p, rand_val, out); break;
        case 1024: fused_top_p_sample_1024<<<1, 1024, 0, s>>>(cand, top_p, rand_val, out); break;
        default: return -1;  // the reference rejects other candidate counts
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
