// Element-wise pieces of the Whisper encoder around its GEMMs (gemm_tc.cu) and attention
// (attn_tc.cu).
//
// layer_norm_rows_kernel: ops.layerNorm (src/ops.zig:355-398) over the 1500 rows of every
//   window (src/encoder.zig:153, 170, 178), one warp per row held in registers: the mean,
//   the population variance about it, inv = 1 / sqrt(var + eps), out = fma((x - mean) * inv,
//   w, b); written as f16 (the operand of the next projection) or f32 (ln_post, in place).
// mel_rows_kernel: the log-mel frames of each 30 s window (src/encoder.zig:125-135 reads
//   mel[c][offset + t]) transposed into f16 rows [1 + t][c] with a zero row on each side, so
//   that row t of the kernel-3 convolution's operand is the three consecutive rows t-1, t,
//   t+1: one strided view, no im2col copy.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace zwg {

// V float4 per lane: n = 128 * V
template <int V, bool OUT_F16>
__global__ void __launch_bounds__(256) layer_norm_rows_kernel(const float* x, size_t n_rows, const float* __restrict__ w,
                                                              const float* __restrict__ b, float eps, void* out) {
    constexpr int N = 128 * V;
    const size_t row = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n_rows) return;
    const float4* xr = reinterpret_cast<const float4*>(x + row * N);
    float4 v[V];
#pragma unroll
    for (int i = 0; i < V; i++) v[i] = xr[lane + 32 * i];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; i++) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    s = warp_sum(s);
    const float mean = __fdiv_rn(s, (float)N);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
        q += (a * a + bb * bb) + (c * c + d * d);
    }
    q = warp_sum(q);
    const float var = __fdiv_rn(q, (float)N);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int j = 4 * (lane + 32 * i);
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w + j));
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b + j));
        const float o0 = fmaf(__fmul_rn(v[i].x - mean, inv), wv.x, bv.x);
        const float o1 = fmaf(__fmul_rn(v[i].y - mean, inv), wv.y, bv.y);
        const float o2 = fmaf(__fmul_rn(v[i].z - mean, inv), wv.z, bv.z);
        const float o3 = fmaf(__fmul_rn(v[i].w - mean, inv), wv.w, bv.w);
        if (OUT_F16) {
            __half2 h0 = __floats2half2_rn(o0, o1), h1 = __floats2half2_rn(o2, o3);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&h0);
            u.y = *reinterpret_cast<uint32_t*>(&h1);
            reinterpret_cast<uint2*>(static_cast<__half*>(out) + row * N)[lane + 32 * i] = u;
        } else {
            reinterpret_cast<float4*>(static_cast<float*>(out) + row * N)[lane + 32 * i] = make_float4(o0, o1, o2, o3);
        }
    }
}

int layer_norm_rows_launch(const float* x, size_t n_rows, int n, const float* w, const float* b, float eps, void* out,
                           bool out_f16, cudaStream_t st) {
    if (n_rows == 0) return 0;
    if (n % 128 || n < 128 || n > 1024) return -1;
    if (((uintptr_t)x | (uintptr_t)w | (uintptr_t)b | (uintptr_t)out) & 15) return -1;
    const size_t blocks = (n_rows + 7) / 8;
    if (blocks > 0x7fffffff) return -1;
    const dim3 grid((unsigned)blocks);
#define ZWG_LN_CASE(V)                                                                                   \
    case V:                                                                                              \
        if (out_f16) layer_norm_rows_kernel<V, true><<<grid, 256, 0, st>>>(x, n_rows, w, b, eps, out);   \
        else layer_norm_rows_kernel<V, false><<<grid, 256, 0, st>>>(x, n_rows, w, b, eps, out);          \
        break;
    switch (n / 128) {
        ZWG_LN_CASE(1)
        ZWG_LN_CASE(2)
        ZWG_LN_CASE(3)
        ZWG_LN_CASE(4)
        ZWG_LN_CASE(5)
        ZWG_LN_CASE(6)
        ZWG_LN_CASE(7)
        ZWG_LN_CASE(8)
        default: return -1;
    }
#undef ZWG_LN_CASE
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

// One block transposes 32 frames x 32 channels through shared memory; blockIdx.z = window.
__global__ void __launch_bounds__(256) mel_rows_kernel(const float* __restrict__ mel, int n_mels, size_t n_len,
                                                       const int* __restrict__ offsets, int n_frames,
                                                       uint16_t* __restrict__ rows) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z;
    const long long off = offsets ? (long long)offsets[b] : (long long)b * n_frames;
    const int t0 = blockIdx.x * 32 - 1;  // row r of the output holds frame r - 1
    const int c0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int cy = ty; cy < 32; cy += 8) {
        const int c = c0 + cy, t = t0 + tx;
        float v = 0.f;
        const long long f = off + t;
        if (c < n_mels && t >= 0 && t < n_frames && f >= 0 && f < (long long)n_len) v = mel[(size_t)c * n_len + f];
        tile[cy][tx] = v;
    }
    __syncthreads();
    uint16_t* out = rows + (size_t)b * (n_frames + 2) * n_mels;
    for (int ry = ty; ry < 32; ry += 8) {
        const int r = blockIdx.x * 32 + ry, c = c0 + tx;
        if (r < n_frames + 2 && c < n_mels) out[(size_t)r * n_mels + c] = __half_as_ushort(__float2half_rn(tile[tx][ry]));
    }
}

int mel_rows_launch(const float* mel, int n_mels, size_t n_len, const int* offsets, int n_batch, int n_frames,
                    uint16_t* rows, cudaStream_t st) {
    if (n_batch == 0) return 0;
    if (n_mels <= 0 || n_frames <= 0 || n_batch > 65535) return -1;
    const dim3 grid((unsigned)((n_frames + 2 + 31) / 32), (unsigned)((n_mels + 31) / 32), (unsigned)n_batch);
    mel_rows_kernel<<<grid, 256, 0, st>>>(mel, n_mels, n_len, offsets, n_frames, rows);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace zwg
