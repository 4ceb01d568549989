// The small kernels of a decode step around the projections and the attention (Qwen2:
// src/llm.zig:168-216, 268-273, 313-321; the Whisper decoder: src/decoder.zig:166-206),
// launched as chained launches (chain.cuh) so each one's start overlaps the end of the
// kernel before it.
//
// rms_norm_kernel: ops.rmsNorm (src/ops.zig:408-425), one CTA per row: the sum of squares
//   (f32, tree order), inv = 1 / sqrt(ss / n + eps) with correctly rounded division and
//   square root, out = x * inv * w as two rounded products in the reference's order.
// layer_norm_kernel: ops.layerNorm (src/ops.zig:355-398), one CTA per row: the mean, then
//   the population variance about it, inv = 1 / sqrt(var + eps), out = fma((x - mean) * inv,
//   w, b) as the reference's vector loop.
// embed_q8_kernel: Q8.row (src/gemm.zig:256-263) for the token of each row: q * scale in
//   f32, bit-identical to the reference; with a positional table the row then adds its
//   position's row, as the Whisper decoder does (src/decoder.zig:172-176). A token outside
//   the vocabulary writes a zero row and sets the device error word.
// greedy_kernel: Model.penalize then Model.argmax (src/llm.zig:313-321, 268-273), one CTA
//   per sequence: the repeat penalty over the last `window` generated tokens (repeats are
//   penalized again, as in the reference), then the first index of the largest logit (NaN
//   never wins; a NaN in column 0 makes the answer 0, as the reference's strict comparison
//   does).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <climits>

#include "chain.cuh"
#include "common.cuh"
#include "kernels.h"

namespace zwg {

__global__ void __launch_bounds__(256) rms_norm_kernel(const float* x, size_t x_stride, int n,
                                                       const float* __restrict__ w, float eps, float* out,
                                                       size_t out_stride) {
    chain_release();
    const int z = chain_wait();
    const float* row = x + blockIdx.x * x_stride + z;
    float* o = out + blockIdx.x * out_stride + z;
    float ss = 0.f;
    for (int j = threadIdx.x * 4; j < n; j += 1024) {
        const float4 v = __ldca(reinterpret_cast<const float4*>(row + j));
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    __shared__ float part[8];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += part[i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    for (int j = threadIdx.x * 4; j < n; j += 1024) {
        const float4 v = __ldca(reinterpret_cast<const float4*>(row + j));
        const float4 g = __ldg(reinterpret_cast<const float4*>(w + j));
        float4 r;
        r.x = __fmul_rn(__fmul_rn(v.x, inv), g.x);
        r.y = __fmul_rn(__fmul_rn(v.y, inv), g.y);
        r.z = __fmul_rn(__fmul_rn(v.z, inv), g.z);
        r.w = __fmul_rn(__fmul_rn(v.w, inv), g.w);
        *reinterpret_cast<float4*>(o + j) = r;
    }
}

__global__ void __launch_bounds__(256) layer_norm_kernel(const float* x, size_t x_stride, int n,
                                                         const float* __restrict__ w, const float* __restrict__ bias,
                                                         float eps, float* out, size_t out_stride) {
    chain_release();
    const int z = chain_wait();
    const float* row = x + blockIdx.x * x_stride + z;
    float* o = out + blockIdx.x * out_stride + z;
    __shared__ float part[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // mean, then the population variance about it (two passes, as the reference)
    float s = 0.f;
    for (int j = threadIdx.x * 4; j < n; j += 1024) {
        const float4 v = __ldca(reinterpret_cast<const float4*>(row + j));
        s += (v.x + v.y) + (v.z + v.w);
    }
    s = warp_sum(s);
    if (lane == 0) part[warp] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += part[i];
    const float mean = __fdiv_rn(tot, (float)n);
    __syncthreads();
    float q = 0.f;
    for (int j = threadIdx.x * 4; j < n; j += 1024) {
        const float4 v = __ldca(reinterpret_cast<const float4*>(row + j));
        const float a = __fsub_rn(v.x, mean), b = __fsub_rn(v.y, mean), c = __fsub_rn(v.z, mean), d = __fsub_rn(v.w, mean);
        q = fmaf(a, a, q);
        q = fmaf(b, b, q);
        q = fmaf(c, c, q);
        q = fmaf(d, d, q);
    }
    q = warp_sum(q);
    if (lane == 0) part[warp] = q;
    __syncthreads();
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) sq += part[i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, (float)n), eps)));
    for (int j = threadIdx.x * 4; j < n; j += 1024) {
        const float4 v = __ldca(reinterpret_cast<const float4*>(row + j));
        const float4 g = __ldg(reinterpret_cast<const float4*>(w + j));
        const float4 h = __ldg(reinterpret_cast<const float4*>(bias + j));
        float4 r;
        r.x = fmaf(__fmul_rn(__fsub_rn(v.x, mean), inv), g.x, h.x);
        r.y = fmaf(__fmul_rn(__fsub_rn(v.y, mean), inv), g.y, h.y);
        r.z = fmaf(__fmul_rn(__fsub_rn(v.z, mean), inv), g.z, h.z);
        r.w = fmaf(__fmul_rn(__fsub_rn(v.w, mean), inv), g.w, h.w);
        *reinterpret_cast<float4*>(o + j) = r;
    }
}

__global__ void __launch_bounds__(256) embed_q8_kernel(const int32_t* tokens, const int8_t* __restrict__ q,
                                                       const float* __restrict__ scales, int n_vocab, int k,
                                                       const float* __restrict__ pe, int pos0, int n_tok,
                                                       float* out, int* err) {
    chain_release();
    const int z = chain_wait();
    const int t = __ldcg(tokens + blockIdx.x + z);
    float* o = out + (size_t)blockIdx.x * k + z;
    if (t < 0 || t >= n_vocab) {
        for (int j = threadIdx.x; j < k; j += blockDim.x) o[j] = 0.f;
        if (threadIdx.x == 0) set_error(err, kErrBounds);
        return;
    }
    const int8_t* qr = q + (size_t)t * k;
    const float* sr = scales + (size_t)t * (k / 32);
    const float* pr = pe ? pe + (size_t)(pos0 + (int)(blockIdx.x % n_tok)) * k : nullptr;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        const float v = __fmul_rn((float)__ldg(qr + j), __ldg(sr + (j >> 5)));
        o[j] = pr ? __fadd_rn(v, __ldg(pr + j)) : v;
    }
}

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

// One CTA per row. The penalty: thread i takes window entry i; the first occurrence of a
// token applies the penalty as many times as the token occurs in the window, in order, so
// the result equals the reference's loop over the window. The argmax: 8 independent 16-byte
// loads per thread per round, then a block reduction keeping the largest value and, among
// equal values, the smallest index.
__global__ void __launch_bounds__(1024) greedy_kernel(float* logits, int n_vocab, const int32_t* recent,
                                                      size_t recent_stride, int n_recent, int window, float penalty,
                                                      int32_t* out, size_t out_stride, int* err) {
    chain_release();
    const int z = chain_wait();
    float* row = logits + (size_t)blockIdx.x * n_vocab + z;
    if (penalty > 1.0f && n_recent > 0) {
        // the window in shared memory (windows longer than kWin are read from global memory)
        constexpr int kWin = 2048;
        __shared__ int win[kWin];
        const int32_t* rc = recent + blockIdx.x * recent_stride + z;
        const int from = n_recent > window ? n_recent - window : 0;
        const int w = n_recent - from;
        const bool in_smem = w <= kWin;
        if (in_smem)
            for (int i = threadIdx.x; i < w; i += blockDim.x) win[i] = __ldcg(rc + from + i);
        __syncthreads();
        for (int i = threadIdx.x; i < w; i += blockDim.x) {
            const int t = in_smem ? win[i] : __ldcg(rc + from + i);
            if (t < 0 || t >= n_vocab) {
                set_error(err, kErrBounds);
                continue;
            }
            bool first = true;
            int count = 1;
            for (int j = 0; j < w; j++) {
                const int u = in_smem ? win[j] : __ldcg(rc + from + j);
                first = first && !(j < i && u == t);
                count += j > i && u == t;
            }
            if (!first) continue;
            float v = __ldcg(row + t);
            for (int c = 0; c < count; c++) v = v > 0.f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
            __stcg(row + t, v);
        }
        __syncthreads();
    }
    float bv = -INFINITY;
    int bi = INT_MAX;
    constexpr int B = 8;
    const bool vec = (n_vocab % 4) == 0 && (((uintptr_t)row) & 15) == 0;
    const int n4 = vec ? n_vocab / 4 : 0;
    const float4* row4 = reinterpret_cast<const float4*>(row);
    for (int base = threadIdx.x; base < n4; base += B * blockDim.x) {
        float4 v[B];
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int j = base + u * blockDim.x;
            v[u] = j < n4 ? __ldcg(row4 + j) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int j = 4 * (base + u * blockDim.x);
            better(bv, bi, v[u].x, j);
            better(bv, bi, v[u].y, j + 1);
            better(bv, bi, v[u].z, j + 2);
            better(bv, bi, v[u].w, j + 3);
        }
    }
    for (int j = 4 * n4 + threadIdx.x; j < n_vocab; j += blockDim.x) better(bv, bi, __ldcg(row + j), j);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        better(bv, bi, ov, oi);
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : INT_MAX;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            better(bv, bi, ov, oi);
        }
        if (lane == 0) {
            const float first = __ldcg(row);
            out[blockIdx.x * out_stride + z] = (isnan(first) || bi == INT_MAX) ? 0 : bi;
        }
    }
}

int rms_norm_launch(const float* x, size_t x_stride, size_t m, size_t n, const float* w, float eps, float* out,
                    size_t out_stride, cudaStream_t st) {
    if (m == 0) return 0;
    return launch_chained(rms_norm_kernel, dim3((unsigned)m), dim3(256), st, x, x_stride, (int)n, w, eps, out,
                          out_stride) == cudaSuccess
               ? 0
               : -1;
}

int layer_norm_launch(const float* x, size_t x_stride, size_t m, size_t n, const float* w, const float* b, float eps,
                      float* out, size_t out_stride, cudaStream_t st) {
    if (m == 0) return 0;
    return launch_chained(layer_norm_kernel, dim3((unsigned)m), dim3(256), st, x, x_stride, (int)n, w, b, eps, out,
                          out_stride) == cudaSuccess
               ? 0
               : -1;
}

int embed_q8_launch(const int32_t* tokens, size_t m, const int8_t* q, const float* scales, size_t n_vocab, size_t k,
                    const float* pe, size_t pos0, size_t n_tok, float* out, int* err, cudaStream_t st) {
    if (m == 0) return 0;
    return launch_chained(embed_q8_kernel, dim3((unsigned)m), dim3(256), st, tokens, q, scales, (int)n_vocab, (int)k,
                          pe, (int)pos0, (int)std::max<size_t>(1, n_tok), out, err) == cudaSuccess
               ? 0
               : -1;
}

int greedy_launch(float* logits, size_t m, size_t n_vocab, const int32_t* recent, size_t recent_stride,
                  size_t n_recent, size_t window, float penalty, int32_t* out, size_t out_stride, int* err,
                  cudaStream_t st) {
    if (m == 0) return 0;
    return launch_chained(greedy_kernel, dim3((unsigned)m), dim3(1024), st, logits, (int)n_vocab, recent,
                          recent_stride, (int)n_recent, (int)window, penalty, out, out_stride, err) == cudaSuccess
               ? 0
               : -1;
}

}  // namespace zwg
