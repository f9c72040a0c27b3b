// ref_argmax.cu - test-side checker, never linked into the product library.
// Launches the reference's argmax_kernel, compiled unchanged from the
// reference's sources (sampling.cu), as CudaFunctions::apply_argmax does
// (src/kernels.rs:322-344): one block of 1024 threads.
#include <cuda_runtime.h>

#include "sampling.cu"

extern "C" int ref_argmax(const void *logits, int vocab, unsigned *out, void *stream) {
    argmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(logits), vocab, out);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
