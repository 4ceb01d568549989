// Small memory-bound kernels around the attention hot path: f32 -> bf16 conversion
// (what a projection epilogue would fuse) and the Qwen2 RoPE + transposed-key cache append
// (src/llm.zig:182-190 scatter, src/llm.zig:221-238 rotation).
#include "common.cuh"
#include "kernels.h"

#include <cuda_bf16.h>

namespace zwg {

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y, size_t n) {
    const size_t n4 = n / 4;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
        __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&a);
        o.y = *reinterpret_cast<uint32_t*>(&b);
        reinterpret_cast<uint2*>(y)[i] = o;
    }
    for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        __nv_bfloat16 h = __float2bfloat16_rn(x[i]);
        y[i] = *reinterpret_cast<uint16_t*>(&h);
    }
}

int f32_to_bf16_launch(const float* x, uint16_t* y, size_t n, cudaStream_t st) {
    if (n == 0) return 0;
    if (((uintptr_t)x & 15) || ((uintptr_t)y & 7)) return -1;
    size_t blocks = (n / 4 + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks == 0) blocks = 1;
    f32_to_bf16_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, y, n);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

// One thread per (item, token, head, pair k < d/2). Query heads are rotated in place; key
// heads are rotated and scattered into the transposed cache; value rows are copied.
// The rotation uses separately rounded products and sums (no fused multiply-add), the
// same f32 operations as the reference's rope (src/llm.zig:230-235), so the cache holds
// the reference's values bit for bit.
__global__ void rope_kt_append_kernel(RopeParams p) {
    const size_t half = p.d / 2;
    const size_t heads = p.n_head + p.n_head_kv;
    const size_t per_item = p.n * heads * half;
    const size_t b = blockIdx.y;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < per_item;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t k = idx % half;
        const size_t hh = (idx / half) % heads;
        const size_t i = idx / half / heads;
        const size_t pos = p.n_past + i;
        const float c = p.cos_tab[pos * half + k];
        const float s = p.sin_tab[pos * half + k];
        if (hh < p.n_head) {
            float* row = p.q + b * p.q_bs + i * (p.n_head * p.d) + hh * p.d;
            const float a = row[k], bb = row[k + half];
            row[k] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, s));
            row[k + half] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(bb, c));
        } else {
            const size_t h = hh - p.n_head;
            const size_t kvw = p.n_head_kv * p.d;
            const float* row = p.k + b * p.kv_bs + i * kvw + h * p.d;
            const float a = row[k], bb = row[k + half];
            float* kt = p.cache_kt + b * p.cache_bs;
            kt[(h * p.d + k) * p.n_ctx + pos] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, s));
            kt[(h * p.d + k + half) * p.n_ctx + pos] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(bb, c));
            const float* vr = p.v + b * p.kv_bs + i * kvw + h * p.d;
            float* vc = p.cache_v + b * p.cache_bs + pos * kvw + h * p.d;
            vc[k] = vr[k];
            vc[k + half] = vr[k + half];
        }
    }
}

int rope_kt_append_launch(const RopeParams& p, size_t n_batch, cudaStream_t st) {
    if (n_batch == 0 || p.n == 0) return 0;
    const size_t per_item = p.n * (p.n_head + p.n_head_kv) * (p.d / 2);
    size_t blocks = (per_item + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    dim3 grid((unsigned)blocks, (unsigned)n_batch);
    rope_kt_append_kernel<<<grid, 256, 0, st>>>(p);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace zwg
