// Q8 weights on the GPU: quantization and the linear layer over int8 blocks.
//
// Reference: gemm.Q8 (src/gemm.zig:188-263): a weight matrix [n][k] stored as int8 with one
// f32 scale per block of 32 along k (scale = absmax / 127); ops.linear (src/ops.zig:280-306)
// -> gemm.ntBlockQ (src/gemm.zig:268-351): out[m][n] = x[m][k] . W[n][k]^T + b[n], each
// block's dot product taken on the int8 values widened to f32 and scaled once per block.
// These are the projections around the attention calls (src/decoder.zig:389-413,
// src/llm.zig:179-216).
//
// q8_quantize_kernel: one warp per block of 32 weights (lane = weight): absmax by a warp
//   max over the bit patterns of |v|, scale = absmax / 127 and q = clamp(round(v * (127 /
//   absmax)), -127, 127) with the reference's f32 operations and round-half-away, so the
//   int8 values and scales are bit-identical to Q8.quantize.
// q8_linear_kernel<MR>: the decode-shaped product (m <= 8 rows of x per launch; larger m in
//   chunks of 8). The weight bytes are the traffic (1.125 B per weight with the scales), so
//   the kernel streams them once: a warp owns 1-4 weight rows, lane l reads 16 (8 for MR = 8)
//   consecutive int8 of each row per step (one 128-bit load, a 512-byte coalesced row
//   segment per warp), widens them to f32 exactly (byte permute into a 2^23 float, then one
//   subtraction), takes the dot with the same k range of every x row (rows in pairs per
//   packed f32x2 FMA) and scales it by the block's scale. Warp shuffles sum the lanes; the
//   bias is added on the way out.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zwg {
namespace q8 {

constexpr int BLOCK = 32;
constexpr int WARPS = 8;  // per CTA
// Weight rows per warp (RW) and k steps unrolled per lane (UNR) are chosen so that each lane
// has about four 16-byte weight loads in flight: with 24-32 resident warps per SM that is
// 50-64 KB per SM, enough to cover the memory latency. Short rows (k <= 512) take 4 rows
// per warp, k <= 1536 two, longer rows one row with 4 steps unrolled. With 4-8 x rows a warp
// takes 4 weight rows, so each x value loaded serves four of them.
__global__ void __launch_bounds__(256) q8_quantize_kernel(const float* __restrict__ w, int n, int k,
                                                          int8_t* __restrict__ q, float* __restrict__ scales) {
    const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // global warp = block
    const int lane = threadIdx.x & 31;
    const int nb = k / BLOCK;
    if (gw >= (long long)n * nb) return;
    const int row = (int)(gw / nb), b = (int)(gw % nb);
    const size_t idx = (size_t)row * k + (size_t)b * BLOCK + lane;
    const float v = w[idx];
    // |v| is non-negative: its bit pattern orders like the value
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
    const float scale = __fdiv_rn(amax, 127.0f);
    const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
    const float r = roundf(__fmul_rn(v, inv));  // half away from zero, as Zig's @round
    q[idx] = (int8_t)fminf(fmaxf(r, -127.f), 127.f);
    if (lane == 0) scales[(size_t)row * nb + b] = scale;
}

// int8 byte j of word u (biased by 0x80) -> float, exactly: 0x4B0000xx is 2^23 + xx.
__device__ __forceinline__ float i8f(uint32_t ub, int j) {
    return __uint_as_float(__byte_perm(ub, 0x4B000000u, 0x7650u | (uint32_t)j)) - 8388736.0f;  // 2^23 + 128
}

template <int MR, int RW>
__global__ void __launch_bounds__(256, MR >= 4 ? 1 : 3) q8_linear_kernel(const float* __restrict__ x, int m, int k,
                                                        const int8_t* __restrict__ wq, const float* __restrict__ ws,
                                                        const float* __restrict__ bias, int n,
                                                        float* __restrict__ out) {
    constexpr int KL = MR >= 8 ? 8 : 16;  // k per lane per step
    constexpr int MP = (MR + 1) / 2;      // x row pairs
    constexpr int UNR = (MR <= 2 && RW == 1) ? 4 : 1;  // k steps unrolled per lane
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * WARPS + warp) * RW;
    if (row0 >= n) return;
    const int nb = k / BLOCK;
    const int8_t* wr[RW];
    const float* sr[RW];
#pragma unroll
    for (int r = 0; r < RW; r++) {
        const int row = min(row0 + r, n - 1);  // rows past n repeat the last row; not stored
        wr[r] = wq + (size_t)row * k;
        sr[r] = ws + (size_t)row * nb;
    }
    float2 acc[RW][MP];
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int p = 0; p < MP; p++) acc[r][p] = make_float2(0.f, 0.f);

#pragma unroll UNR
    for (int k0 = lane * KL; k0 < k; k0 += 32 * KL) {
        // x rows for this lane's k range
        float xv[MR][KL];
#pragma unroll
        for (int mr = 0; mr < MR; mr++) {
            const int row = mr < m ? mr : 0;
#pragma unroll
            for (int i = 0; i < KL; i += 4) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(x + (size_t)row * k + k0 + i));
                xv[mr][i] = mr < m ? f.x : 0.f;
                xv[mr][i + 1] = mr < m ? f.y : 0.f;
                xv[mr][i + 2] = mr < m ? f.z : 0.f;
                xv[mr][i + 3] = mr < m ? f.w : 0.f;
            }
        }
#pragma unroll
        for (int r = 0; r < RW; r++) {
            uint32_t wv[KL / 4];
            if constexpr (KL == 16) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(wr[r] + k0));
                wv[0] = u.x; wv[1] = u.y; wv[2] = u.z; wv[3] = u.w;
            } else {
                const uint2 u = __ldg(reinterpret_cast<const uint2*>(wr[r] + k0));
                wv[0] = u.x; wv[1] = u.y;
            }
            const float sc = __ldg(sr[r] + k0 / BLOCK);
            float2 t[MP];
#pragma unroll
            for (int p = 0; p < MP; p++) t[p] = make_float2(0.f, 0.f);
#pragma unroll
            for (int wd = 0; wd < KL / 4; wd++) {
                const uint32_t ub = wv[wd] ^ 0x80808080u;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float qf = i8f(ub, j);
                    const int i = wd * 4 + j;
#pragma unroll
                    for (int p = 0; p < MP; p++) {
                        const float xb = (2 * p + 1 < MR) ? xv[2 * p + 1][i] : 0.f;
                        t[p] = __ffma2_rn(make_float2(xv[2 * p][i], xb), make_float2(qf, qf), t[p]);
                    }
                }
            }
            // the block's scale once per partial dot (the reference scales whole blocks)
#pragma unroll
            for (int p = 0; p < MP; p++) acc[r][p] = __ffma2_rn(t[p], make_float2(sc, sc), acc[r][p]);
        }
    }
    // sum over the lanes; every lane ends with every total
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int p = 0; p < MP; p++)
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                acc[r][p].x += __shfl_xor_sync(0xffffffffu, acc[r][p].x, off);
                acc[r][p].y += __shfl_xor_sync(0xffffffffu, acc[r][p].y, off);
            }
    // lane r * MR + mr writes out[mr][row0 + r]
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int mr = 0; mr < MR; mr++) {
            if (lane == r * MR + mr && mr < m && row0 + r < n) {
                const float v = (mr & 1) ? acc[r][mr >> 1].y : acc[r][mr >> 1].x;
                out[(size_t)mr * n + row0 + r] = bias ? v + bias[row0 + r] : v;
            }
        }
}

}  // namespace q8

int q8_quantize_launch(const float* w, size_t n, size_t k, int8_t* q, float* scales, cudaStream_t st) {
    const long long blocks = (long long)n * (k / q8::BLOCK);
    if (blocks == 0) return 0;
    const long long grid = (blocks + 7) / 8;
    if (grid > 0x7fffffffll) return -1;
    q8::q8_quantize_kernel<<<(unsigned)grid, 256, 0, st>>>(w, (int)n, (int)k, q, scales);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int q8_linear_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias,
                     size_t n, float* out, cudaStream_t st) {
    if (m == 0 || n == 0) return 0;
    const int rw = k <= 512 ? 4 : k <= 1536 ? 2 : 1;  // weight rows per warp for 1-2 x rows
    for (size_t m0 = 0; m0 < m; m0 += 8) {
        const int mc = (int)std::min<size_t>(8, m - m0);
        const float* xc = x + m0 * k;
        float* oc = out + m0 * n;
        const int r = mc <= 2 ? rw : 4;
        const unsigned grid = (unsigned)((n + q8::WARPS * r - 1) / (q8::WARPS * r));
        const int ik = (int)k, in = (int)n;
        if (mc == 1) {
            if (r == 4) q8::q8_linear_kernel<1, 4><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
            else if (r == 2) q8::q8_linear_kernel<1, 2><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
            else q8::q8_linear_kernel<1, 1><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
        } else if (mc == 2) {
            if (r == 4) q8::q8_linear_kernel<2, 4><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
            else if (r == 2) q8::q8_linear_kernel<2, 2><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
            else q8::q8_linear_kernel<2, 1><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
        } else if (mc <= 4) {
            q8::q8_linear_kernel<4, 4><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
        } else {
            q8::q8_linear_kernel<8, 4><<<grid, 256, 0, st>>>(xc, mc, ik, wq, ws, bias, in, oc);
        }
        if (cudaPeekAtLastError() != cudaSuccess) return -1;
    }
    return 0;
}

}  // namespace zwg
