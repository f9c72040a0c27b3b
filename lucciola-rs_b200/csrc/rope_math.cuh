// rope_math.cuh - the rotate-half RoPE arithmetic of src/kernels/rope.cu:22-53,
// written so that it rounds exactly as the reference kernel does.
//
// The reference computes in fp32 with the CUDA compiler's default FMA
// contraction. The two expressions x1*c - x2*s and x1*s + x2*c are written here
// with explicit round-to-nearest intrinsics in the contraction form that
// reproduces the reference kernel's results bit for bit (pinned by comparing
// outputs on a B200; the modes are those of oracle/lc_oracle.h). Shared by the
// standalone append kernel and the fused append + decode kernel.
#pragma once

#ifndef LC_ROPE_SUB_MODE
#define LC_ROPE_SUB_MODE 1  // x1*c - x2*s  ->  fma(x1, c, -(x2*s))
#endif
#ifndef LC_ROPE_ADD_MODE
#define LC_ROPE_ADD_MODE 1  // x1*s + x2*c  ->  fma(x1, s, x2*c)
#endif

namespace lc {

__device__ __forceinline__ float rot_sub(float x1, float c, float x2, float s) {
#if LC_ROPE_SUB_MODE == 1
    return __fmaf_rn(x1, c, -__fmul_rn(x2, s));
#elif LC_ROPE_SUB_MODE == 2
    return __fmaf_rn(-x2, s, __fmul_rn(x1, c));
#else
    return __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
#endif
}

__device__ __forceinline__ float rot_add(float x1, float s, float x2, float c) {
#if LC_ROPE_ADD_MODE == 1
    return __fmaf_rn(x1, s, __fmul_rn(x2, c));
#elif LC_ROPE_ADD_MODE == 2
    return __fmaf_rn(x2, c, __fmul_rn(x1, s));
#else
    return __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
#endif
}

}  // namespace lc
