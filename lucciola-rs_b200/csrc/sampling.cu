// sampling.cu - token selection from the logits of a batch of sequences:
//   lc_argmax        greedy: the largest logit of each row        (src/kernels/sampling.cu,
//                    src/kernels.rs:322-344: one sequence, one block of 1024 threads)
//   lc_sample_top_p  top-k candidates, softmax, top-p cutoff and an inverse-CDF
//                    draw with a caller-given uniform number per row
//                    (src/kernels/sampling_optimized.cu, src/kernels.rs:346-490)
//
// The reference runs one sequence per launch; here one launch covers the batch
// (a block per row, or per (row, vocabulary partition)), reads the bf16 logits
// (argmax with 16-byte loads where rows are aligned) and keeps the candidates in
// a caller workspace. Results equal the reference's: the candidate set is that
// of its 32-partition top-k filter, and ties are broken in the order its
// reductions break them, stated as explicit keys:
//   argmax:      larger value, then lower i % 1024 (the reference thread), then
//                lower i;
//   top-k:       per partition of [p*V/32, (p+1)*V/32): larger value, then the
//                reference warp / lane order of its shfl_down trees (bit-reversed
//                warp, then bit-reversed lane, of thread i % 256), then lower i.
// A logit must exceed -1e30 to be chosen (the reference's starting value, kept
// with a strict comparison); a row with none gives index 0xffffffff (argmax).
#include <climits>

#include "lc_common.cuh"
#include "lc_host.h"

namespace lc {
namespace {

constexpr float kNone = -1e30f;

struct Cand {
    float v;
    int i;  // -1: none
};

// argmax order: is a before b?
__device__ __forceinline__ bool argmax_before(const Cand &a, const Cand &b) {
    if (a.i < 0) return false;
    if (b.i < 0) return a.v > b.v;
    if (a.v != b.v) return a.v > b.v;
    const int ta = a.i & 1023, tb = b.i & 1023;
    return ta != tb ? ta < tb : a.i < b.i;
}

__device__ __forceinline__ int bitrev5(int x) { return (int)(__brev((unsigned)x) >> 27); }

// top-k filter order within a partition (i: partition-local index).
__device__ __forceinline__ bool topk_before(const Cand &a, const Cand &b) {
    if (a.i < 0) return false;
    if (b.i < 0) return a.v > b.v;
    if (a.v != b.v) return a.v > b.v;
    const int ta = a.i & 255, tb = b.i & 255;
    const int pa = bitrev5(ta >> 5) * 32 + bitrev5(ta & 31);
    const int pb = bitrev5(tb >> 5) * 32 + bitrev5(tb & 31);
    return pa != pb ? pa < pb : a.i < b.i;
}

template <bool (*Before)(const Cand &, const Cand &)>
__device__ __forceinline__ Cand warp_best(Cand c) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Cand d;
        d.v = __shfl_xor_sync(0xffffffffu, c.v, o);
        d.i = __shfl_xor_sync(0xffffffffu, c.i, o);
        if (Before(d, c)) c = d;
    }
    return c;
}

// Best of the block (all threads get it); `red` holds one Cand per warp.
template <bool (*Before)(const Cand &, const Cand &)>
__device__ __forceinline__ Cand block_best(Cand c, Cand *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    c = warp_best<Before>(c);
    if (lane == 0) red[warp] = c;
    __syncthreads();
    Cand r = lane < nw ? red[lane] : Cand{kNone, -1};
    r = warp_best<Before>(r);
    __syncthreads();  // red may be reused by the caller
    return r;
}

// ------------------------------------------------------------------ argmax --
__global__ void __launch_bounds__(1024) argmax_kernel(const bf16 *logits, int64_t stride, int vocab,
                                                      unsigned *out, int vec) {
    __shared__ Cand red[32];
    const bf16 *row = logits + (int64_t)blockIdx.x * stride;
    Cand best{kNone, -1};
    const int n8 = vec ? vocab >> 3 : 0;  // rows not 16-byte aligned: element by element
    for (int c = threadIdx.x; c < n8; c += blockDim.x) {
        const uint4 u = reinterpret_cast<const uint4 *>(row)[c];
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const Cand a{__low2float(h[e]), 8 * c + 2 * e};
            const Cand b{__high2float(h[e]), 8 * c + 2 * e + 1};
            if (argmax_before(a, best)) best = a;
            if (argmax_before(b, best)) best = b;
        }
    }
    for (int i = 8 * n8 + threadIdx.x; i < vocab; i += blockDim.x) {
        const Cand a{__bfloat162float(row[i]), i};
        if (argmax_before(a, best)) best = a;
    }
    best = block_best<argmax_before>(best, red);
    if (threadIdx.x == 0) out[blockIdx.x] = (unsigned)best.i;
}

// ------------------------------------------------------------ top-k filter --
// Block (p, b): partition p of row b, 256 threads (the reference's thread
// count, which the tie order refers to). Element i belongs to thread i % 256;
// each thread keeps the best of its elements, so after a pick only the
// winner's thread rescans.
__global__ void __launch_bounds__(256) topk_filter_kernel(const bf16 *logits, int64_t stride,
                                                          int vocab, int kpb, int *keys,
                                                          float *vals) {
    extern __shared__ float part[];
    __shared__ Cand red[8];
    const int p = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int start = (int)((long long)p * vocab / 32);
    const int end = (int)((long long)(p + 1) * vocab / 32);
    const int n = end - start;
    if (n <= 0) return;  // the reference writes nothing for an empty partition
    const bf16 *row = logits + (int64_t)b * stride + start;
    for (int i = tid; i < n; i += 256) part[i] = __bfloat162float(row[i]);
    __syncthreads();
    auto rescan = [&]() {
        Cand c{kNone, -1};
        for (int i = tid; i < n; i += 256)
            if (part[i] > c.v) c = Cand{part[i], i};
        return c;
    };
    Cand mine = rescan();
    const int ncand = 32 * kpb;
    int *krow = keys + (int64_t)b * ncand + p * kpb;
    float *vrow = vals + (int64_t)b * ncand + p * kpb;
    for (int k = 0; k < kpb; ++k) {
        const Cand w = block_best<topk_before>(mine, red);
        if (tid == 0) {
            krow[k] = start + w.i;  // start - 1 when the partition is exhausted
            vrow[k] = w.i >= 0 ? w.v : kNone;
        }
        if (w.i >= 0 && (w.i & 255) == tid) {
            part[w.i] = kNone;
            mine = rescan();
        }
    }
}

// ------------------------------------------------------- sort and sample --
// One block of n threads per row: the reference's bitonic network (descending,
// equal values keep its order), softmax over the candidates, the top-p cutoff
// (the first cumulative probability >= top_p) and the draw: the candidate
// whose cumulative interval holds rand * cutoff. No winner (rounding at the
// top) leaves out[b] as it was, as the reference does.
__global__ void __launch_bounds__(1024) sort_sample_kernel(const int *keys, const float *vals,
                                                           int n, const float *top_p,
                                                           const float *rand_vals,
                                                           unsigned *out) {
    extern __shared__ unsigned char dyn[];
    float *sv = reinterpret_cast<float *>(dyn);
    int *sk = reinterpret_cast<int *>(sv + n);
    __shared__ float warp_sum[32];
    __shared__ float s_total, s_cutoff;
    const int b = blockIdx.x, t = threadIdx.x;
    sv[t] = vals[(int64_t)b * n + t];
    sk[t] = keys[(int64_t)b * n + t];
    __syncthreads();
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int o = t ^ j;
            if (o > t) {
                const bool swap = (t & k) == 0 ? sv[t] < sv[o] : sv[t] > sv[o];
                if (swap) {
                    const float fv = sv[t];
                    const int fk = sk[t];
                    sv[t] = sv[o], sk[t] = sk[o];
                    sv[o] = fv, sk[o] = fk;
                }
            }
            __syncthreads();
        }
    }
    const float e = expf(sv[t] - sv[0]);
    // total: warp sums, then the warps' sums in order
    const int warp = t >> 5, lane = t & 31, nw = n >> 5;
    float ws = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
    if (lane == 0) warp_sum[warp] = ws;
    if (t == 0) s_cutoff = 1.0f;
    __syncthreads();
    if (t == 0) {
        float tot = 0.f;
        for (int w = 0; w < nw; ++w) tot += warp_sum[w];
        s_total = tot;
    }
    __syncthreads();
    const float prob = e / s_total;
    // inclusive scan: within the warp, then the preceding warps' totals
    float c = prob;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, c, o);
        if (lane >= o) c += y;
    }
    __syncthreads();
    if (lane == 31) warp_sum[warp] = c;
    __syncthreads();
    float before = 0.f;
    for (int w = 0; w < warp; ++w) before += warp_sum[w];
    const float cdf = before + c;
    const float prev = cdf - prob;
    const float tp = top_p[b];
    if (prev < tp && cdf >= tp) s_cutoff = cdf;
    __syncthreads();
    const float target = rand_vals[b] * s_cutoff;
    if (cdf >= target && prev < target) out[b] = (unsigned)sk[t];
}

bool candidates_ok(int top_k, int *n) {
    if (top_k < 32) return false;
    const int c = 32 * (top_k / 32);
    if (c > 1024 || (c & (c - 1))) return false;  // the reference's 32 .. 1024 kernels
    *n = c;
    return true;
}

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" int lc_argmax(const void *logits, int64_t row_stride, int vocab, int batch,
                         unsigned *out_idx, lc_stream_t stream) {
    if (!logits || !out_idx || vocab <= 0 || batch < 0 || row_stride < vocab)
        return LC_ERR_INVALID_ARGUMENT;
    if (batch == 0) return LC_OK;
    const int vec = aligned16(logits) && (row_stride & 7) == 0;
    argmax_kernel<<<batch, 1024, 0, as_stream(stream)>>>((const bf16 *)logits, row_stride, vocab,
                                                          out_idx, vec);
    return launch_status();
}

extern "C" size_t lc_sample_workspace_size(int batch, int top_k) {
    int n = 0;
    if (batch <= 0 || !candidates_ok(top_k, &n)) return 0;
    return (size_t)batch * n * 8;
}

extern "C" int lc_sample_top_p(const void *logits, int64_t row_stride, int vocab, int batch,
                               int top_k, const float *top_p, const float *rand_vals,
                               unsigned *out_idx, void *workspace, size_t workspace_bytes,
                               lc_stream_t stream) {
    if (!logits || !top_p || !rand_vals || !out_idx || vocab <= 0 || batch < 0 ||
        row_stride < vocab)
        return LC_ERR_INVALID_ARGUMENT;
    int n = 0;
    if (!candidates_ok(top_k, &n) || vocab < 32) return LC_ERR_UNSUPPORTED_SHAPE;
    if (batch == 0) return LC_OK;
    if (!workspace || workspace_bytes < lc_sample_workspace_size(batch, top_k))
        return LC_ERR_WORKSPACE_TOO_SMALL;
    if (batch > 65535) return LC_ERR_INVALID_ARGUMENT;
    const int kpb = top_k / 32;
    int *keys = (int *)workspace;
    float *vals = (float *)(keys + (size_t)batch * n);
    const size_t part_bytes = ((size_t)vocab / 32 + 1) * 4;
    if (part_bytes > 227 * 1024) return LC_ERR_UNSUPPORTED_SHAPE;
    int rc = ensure_smem_attr((const void *)topk_filter_kernel, (int)part_bytes);
    if (rc) return rc;
    cudaStream_t s = as_stream(stream);
    topk_filter_kernel<<<dim3(32, batch), 256, part_bytes, s>>>((const bf16 *)logits, row_stride,
                                                                vocab, kpb, keys, vals);
    if (launch_status() != LC_OK) return LC_ERR_CUDA;
    sort_sample_kernel<<<batch, n, (size_t)n * 8, s>>>(keys, vals, n, top_p, rand_vals, out_idx);
    return launch_status();
}
