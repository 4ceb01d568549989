// Q8 weights on the GPU: quantization and the linear layers over int8 blocks.
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
// q8_linear_kernel<MR, RW, KS, UNR>: the decode-shaped product (m <= 8 rows of x per launch;
//   9-15 rows in chunks of 8; 16 or more rows go to the register-tiled product of
//   q8_gemm.cu, pairs included). The weight bytes are the traffic (1.125 B per weight with the
//   scales), so the kernel streams them once: a warp owns RW weight rows over 1/KS of k
//   (KS warps of a CTA share a row set and add their partial sums through shared memory in
//   a fixed order), lane l reads 16 (8 for MR = 8) consecutive int8 of each row per step
//   (one 128-bit load, a 512-byte coalesced row segment per warp) with UNR steps in flight,
//   widens them to f32 exactly (byte permute into a 2^23 float, then one packed
//   subtraction), takes the dot with the same k range of every x row (packed f32x2 FMAs)
//   and scales it by the block's scale. Warp shuffles sum the lanes; the bias is added on
//   the way out; the epilogue then stores, adds into `out` (the residual: ops.linear then
//   ops.add, src/llm.zig:203-204, 209-210; src/decoder.zig:185-186) or applies GELU
//   (ops.linear then ops.gelu, src/decoder.zig:197-198).
// q8_pair_kernel<MR, RP, KS, UNR, EPI>: the same dot products for two matrices' rows at once, a warp
//   owning RP pairs of rows whose outputs one epilogue combines:
//   - PAIR_ROPE: rows i and i + d/2 of one head of the q, k or v projection
//     (src/llm.zig:179-181): bias, then the NeoX rotation at position n_past + t
//     (src/llm.zig:221-238) for q and k; q goes to its output, k into the transposed cache
//     and v into the value cache (src/llm.zig:182-190). One launch replaces three linears,
//     two rope passes and the scatter.
//   - PAIR_SILU: row j of w_gate and of w_up (src/llm.zig:206-208): silu(g) * u
//     (ops.siluMul, src/ops.zig:435-440). One launch replaces two linears and the product.
//
// Launch chaining: every Q8 kernel is launched as a programmatic dependent launch. It
// first hints its own weight rows into L2 (they are constants of the model, not outputs
// of the kernel before it), lets the next kernel in the stream launch, and only then
// waits for the previous kernel's results (griddepcontrol.wait) before reading x or
// writing anything. In a chain of projections each kernel's weight stream therefore
// starts while its predecessor is still running.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "chain.cuh"
#include "common.cuh"
#include "kernels.h"

namespace zwg {
namespace q8 {

constexpr int BLOCK = 32;
constexpr int WARPS = 8;  // per CTA
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

// Bytes of a weight row one warp step covers: 32 lanes x KL int8.
template <int MR>
constexpr int step_bytes() { return 32 * (MR >= 8 ? 8 : 16); }

// k range [kbeg, kend) of split ks of KS: whole warp steps, the last split possibly short
// or empty.
template <int MR, int KS>
__device__ __forceinline__ void split_range(int k, int ks, int& kbeg, int& kend) {
    constexpr int S = step_bytes<MR>();
    const int steps = (k + S - 1) / S;
    const int per = (steps + KS - 1) / KS;
    kbeg = min(k, ks * per * S);
    kend = min(k, kbeg + per * S);
}

// Programmatic dependent launch: hint this warp's part of its weight rows and scales into
// L2, let the next grid launch, then wait until the previous grid's writes are visible.
// Safe whether or not the grid was launched as a dependent (the wait returns at once when
// it was not). Returns the opaque zero of chain_wait, added to the row pointers here and to
// x by the callers.
template <int RW>
__device__ __forceinline__ int chain_prologue(const int8_t* (&wr)[RW], const float* (&sr)[RW], int kbeg, int kend,
                                              int lane) {
    if (kend > kbeg) {
#pragma unroll
        for (int r = 0; r < RW; r++) {
            const uintptr_t a = (uintptr_t)(wr[r] + kbeg), w0 = a & ~(uintptr_t)127;
            const int wl = (int)((a + (kend - kbeg) - 1 - w0) >> 7) + 1;  // 128-byte lines of the range
            for (int i = lane; i < wl; i += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(w0 + ((uintptr_t)i << 7)));
            const uintptr_t b = (uintptr_t)(sr[r] + kbeg / BLOCK), s0 = b & ~(uintptr_t)127;
            const int sl = (int)((b + (kend - kbeg) / BLOCK * 4 - 1 - s0) >> 7) + 1;
            for (int i = lane; i < sl; i += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(s0 + ((uintptr_t)i << 7)));
        }
    }
    chain_release();
    const int z = chain_wait();
#pragma unroll
    for (int r = 0; r < RW; r++) {
        wr[r] += z;
        sr[r] += z;
    }
    return z;
}

// The dot products of RW weight rows with MR rows of x over k in [kbeg, kend) (rows >= m
// read row 0 and count as zero), summed over the warp: every lane ends with every total.
// acc[r][p] holds x rows 2p and 2p + 1 against weight row r (with one x row, acc[r][0].x
// holds the total). The weight loads of UNR steps are issued together before any
// arithmetic, so a warp whose range fits in UNR steps waits for memory once. Per 4 weights
// the widening costs 4 byte permutes and 2 packed subtractions; with one x row the FMAs run
// over pairs of consecutive weights, with two over the x rows.
template <int MR, int RW, int UNR>
__device__ __forceinline__ void dot_rows(const float* x, int m, int k, int kbeg, int kend,
                                         const int8_t* const (&wr)[RW], const float* const (&sr)[RW], int lane,
                                         float2 (&acc)[RW][(MR + 1) / 2]) {
    constexpr int KL = MR >= 8 ? 8 : 16;  // k per lane per step
    constexpr int S = 32 * KL;
    constexpr int MP = (MR + 1) / 2;  // x row pairs
    const float2 magic = make_float2(8388736.0f, 8388736.0f);  // 2^23 + 128
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int p = 0; p < MP; p++) acc[r][p] = make_float2(0.f, 0.f);

    for (int kb = kbeg + lane * KL; kb < kend; kb += UNR * S) {
        uint32_t wv[UNR][RW][KL / 4];
        float sc[UNR][RW];
#pragma unroll
        for (int u = 0; u < UNR; u++) {
            const int k0 = kb + u * S;
#pragma unroll
            for (int r = 0; r < RW; r++) {
                if (k0 < kend) {
                    if constexpr (KL == 16) {
                        const uint4 w = __ldg(reinterpret_cast<const uint4*>(wr[r] + k0));
                        wv[u][r][0] = w.x; wv[u][r][1] = w.y; wv[u][r][2] = w.z; wv[u][r][3] = w.w;
                    } else {
                        const uint2 w = __ldg(reinterpret_cast<const uint2*>(wr[r] + k0));
                        wv[u][r][0] = w.x; wv[u][r][1] = w.y;
                    }
                    sc[u][r] = __ldg(sr[r] + k0 / BLOCK);
                } else {
#pragma unroll
                    for (int j = 0; j < KL / 4; j++) wv[u][r][j] = 0;
                    sc[u][r] = 0.f;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < UNR; u++) {
            const int k0 = kb + u * S;
            if (k0 >= kend) break;
            // x rows for this lane's k range
            float xv[MR][KL];
#pragma unroll
            for (int mr = 0; mr < MR; mr++) {
                const int row = mr < m ? mr : 0;
#pragma unroll
                for (int i = 0; i < KL; i += 4) {
                    const float4 f = __ldca(reinterpret_cast<const float4*>(x + (size_t)row * k + k0 + i));
                    xv[mr][i] = mr < m ? f.x : 0.f;
                    xv[mr][i + 1] = mr < m ? f.y : 0.f;
                    xv[mr][i + 2] = mr < m ? f.z : 0.f;
                    xv[mr][i + 3] = mr < m ? f.w : 0.f;
                }
            }
#pragma unroll
            for (int r = 0; r < RW; r++) {
                float2 t[MP];
#pragma unroll
                for (int p = 0; p < MP; p++) t[p] = make_float2(0.f, 0.f);
#pragma unroll
                for (int wd = 0; wd < KL / 4; wd++) {
                    const uint32_t ub = wv[u][r][wd] ^ 0x80808080u;
                    // q + 2^23 + 128 for the four bytes, exact; one packed subtraction per pair
                    const float2 q01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(ub, 0x4B000000u, 0x7650u)),
                                                              __uint_as_float(__byte_perm(ub, 0x4B000000u, 0x7651u))),
                                                  make_float2(-magic.x, -magic.y));
                    const float2 q23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(ub, 0x4B000000u, 0x7652u)),
                                                              __uint_as_float(__byte_perm(ub, 0x4B000000u, 0x7653u))),
                                                  make_float2(-magic.x, -magic.y));
                    const int i = wd * 4;
                    if constexpr (MR == 1) {
                        t[0] = __ffma2_rn(make_float2(xv[0][i], xv[0][i + 1]), q01, t[0]);
                        t[0] = __ffma2_rn(make_float2(xv[0][i + 2], xv[0][i + 3]), q23, t[0]);
                    } else {
#pragma unroll
                        for (int p = 0; p < MP; p++) {
                            const bool two = 2 * p + 1 < MR;
                            t[p] = __ffma2_rn(make_float2(xv[2 * p][i], two ? xv[2 * p + 1][i] : 0.f),
                                              make_float2(q01.x, q01.x), t[p]);
                            t[p] = __ffma2_rn(make_float2(xv[2 * p][i + 1], two ? xv[2 * p + 1][i + 1] : 0.f),
                                              make_float2(q01.y, q01.y), t[p]);
                            t[p] = __ffma2_rn(make_float2(xv[2 * p][i + 2], two ? xv[2 * p + 1][i + 2] : 0.f),
                                              make_float2(q23.x, q23.x), t[p]);
                            t[p] = __ffma2_rn(make_float2(xv[2 * p][i + 3], two ? xv[2 * p + 1][i + 3] : 0.f),
                                              make_float2(q23.y, q23.y), t[p]);
                        }
                    }
                }
                // the block's scale once per partial dot (the reference scales whole blocks)
                const float c = sc[u][r];
                if constexpr (MR == 1) {
                    acc[r][0].x = fmaf(t[0].x + t[0].y, c, acc[r][0].x);
                } else {
#pragma unroll
                    for (int p = 0; p < MP; p++) acc[r][p] = __ffma2_rn(t[p], make_float2(c, c), acc[r][p]);
                }
            }
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
                if constexpr (MR > 1) acc[r][p].y += __shfl_xor_sync(0xffffffffu, acc[r][p].y, off);
            }
}

// Sum the KS k-splits of each row slot in split order (the same order every run), leaving
// the totals in the slot's first warp (warp % KS == 0). Every warp of the CTA calls it.
template <int MR, int RW, int KS>
__device__ __forceinline__ void reduce_splits(float2 (&acc)[RW][(MR + 1) / 2], int warp, int lane) {
    if constexpr (KS > 1) {
        constexpr int MP = (MR + 1) / 2;
        __shared__ float2 red[WARPS][RW][MP];
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < RW; r++)
#pragma unroll
                for (int p = 0; p < MP; p++) red[warp][r][p] = acc[r][p];
        }
        __syncthreads();
        if (warp % KS == 0) {
#pragma unroll
            for (int r = 0; r < RW; r++)
#pragma unroll
                for (int p = 0; p < MP; p++) {
                    float2 t = red[warp][r][p];
#pragma unroll
                    for (int j = 1; j < KS; j++) {
                        t.x += red[warp + j][r][p].x;
                        t.y += red[warp + j][r][p].y;
                    }
                    acc[r][p] = t;
                }
        }
    }
}

// ggml's GELU, the tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) with the
// reference's operation order (src/ops.zig:312-327); tanh is CUDA's tanhf.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(u)));
}

template <int MR, int RW, int KS, int UNR>
__global__ void __launch_bounds__(256, MR >= 4 ? 1 : (RW * UNR >= 8 || (MR == 2 && RW >= 4)) ? 2 : 3) q8_linear_kernel(const float* x, int m, int k,
                                                        const int8_t* __restrict__ wq, const float* __restrict__ ws,
                                                        const float* __restrict__ bias, int n, int mode,
                                                        float* out) {
    constexpr int MP = (MR + 1) / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = warp % KS;
    const int row0 = (blockIdx.x * (WARPS / KS) + warp / KS) * RW;
    const int nb = k / BLOCK;
    int kbeg, kend;
    split_range<MR, KS>(k, ks, kbeg, kend);
    const int8_t* wr[RW];
    const float* sr[RW];
#pragma unroll
    for (int r = 0; r < RW; r++) {
        const int row = min(row0 + r, n - 1);  // rows past n repeat the last row; not stored
        wr[r] = wq + (size_t)row * k;
        sr[r] = ws + (size_t)row * nb;
    }
    const int z = chain_prologue<RW>(wr, sr, kbeg, kend, lane);
    // blockIdx.y walks chunks of MR rows of x (one launch for all full chunks)
    x += z + (size_t)blockIdx.y * MR * k;
    out += z + (size_t)blockIdx.y * MR * n;
    float2 acc[RW][MP];
    dot_rows<MR, RW, UNR>(x, m, k, kbeg, kend, wr, sr, lane, acc);
    reduce_splits<MR, RW, KS>(acc, warp, lane);
    if (ks != 0 || row0 >= n) return;
    // lane r * MR + mr writes out[mr][row0 + r]
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int mr = 0; mr < MR; mr++) {
            if (lane == r * MR + mr && mr < m && row0 + r < n) {
                float v = (mr & 1) ? acc[r][mr >> 1].y : acc[r][mr >> 1].x;
                if (bias) v = __fadd_rn(v, bias[row0 + r]);
                float* o = out + (size_t)mr * n + row0 + r;
                if (mode == LIN_ADD) v = __fadd_rn(__ldcg(o), v);
                else if (mode == LIN_GELU) v = gelu_tanh(v);
                *o = v;
            }
        }
}

template <int MR, int RP, int KS, int UNR, int EPI>
__global__ void __launch_bounds__(256, MR >= 4 ? 1 : (2 * RP * UNR >= 8 || (MR == 2 && RP >= 2)) ? 2 : 3) q8_pair_kernel(const PairParams p) {
    constexpr int RW = 2 * RP;
    constexpr int MP = (MR + 1) / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = warp % KS;
    const int pair0 = (blockIdx.x * (WARPS / KS) + warp / KS) * RP;
    const int k = p.k, nb = k / BLOCK;
    int kbeg, kend;
    split_range<MR, KS>(k, ks, kbeg, kend);
    // rows of the two matrices this warp reads: r < RP the first of each pair, r >= RP the second
    int sec = 0, head = 0, i0 = 0;
    const int8_t* wr[RW];
    const float* sr[RW];
    {
        const int pc = min(pair0, p.n_pairs - 1);  // pairs past the end repeat the last; not stored
        int ra, rb, ma, mb;
        if (EPI == PAIR_ROPE) {
            const int half = p.d >> 1;
            const int hh = pc / half;
            i0 = pc - hh * half;
            sec = hh < p.n_head ? 0 : hh < p.n_head + p.n_head_kv ? 1 : 2;
            head = sec == 0 ? hh : sec == 1 ? hh - p.n_head : hh - p.n_head - p.n_head_kv;
            ra = head * p.d + i0;
            rb = ra + half;
            ma = mb = sec;
        } else {
            i0 = pc;
            ra = rb = pc;
            ma = 0;
            mb = 1;
        }
        const int n_rows_a = EPI == PAIR_ROPE ? (sec == 0 ? p.n_head : p.n_head_kv) * p.d : p.n_pairs;
#pragma unroll
        for (int r = 0; r < RP; r++) {
            const int a = min(ra + r, n_rows_a - 1), b = min(rb + r, n_rows_a - 1);
            wr[r] = p.wq[ma] + (size_t)a * k;
            sr[r] = p.ws[ma] + (size_t)a * nb;
            wr[RP + r] = p.wq[mb] + (size_t)b * k;
            sr[RP + r] = p.ws[mb] + (size_t)b * nb;
        }
    }
    const int z = chain_prologue<RW>(wr, sr, kbeg, kend, lane);
    float2 acc[RW][MP];
    dot_rows<MR, RW, UNR>(p.x + z, p.m, k, kbeg, kend, wr, sr, lane, acc);
    reduce_splits<MR, RW, KS>(acc, warp, lane);
    if (ks != 0 || pair0 >= p.n_pairs) return;

    // lane rp * MR + mr finishes pair pair0 + rp for x row mr
    float va = 0.f, vb = 0.f;
    int rp_sel = -1, mr_sel = 0;
#pragma unroll
    for (int rp = 0; rp < RP; rp++)
#pragma unroll
        for (int mr = 0; mr < MR; mr++)
            if (lane == rp * MR + mr) {
                va = (mr & 1) ? acc[rp][mr >> 1].y : acc[rp][mr >> 1].x;
                vb = (mr & 1) ? acc[RP + rp][mr >> 1].y : acc[RP + rp][mr >> 1].x;
                rp_sel = rp;
                mr_sel = mr;
            }
    if (rp_sel < 0 || mr_sel >= p.m || pair0 + rp_sel >= p.n_pairs) return;
    const int tok = p.m0 + mr_sel;  // row of x over the whole call: sequence * n_tok + t
    if (EPI == PAIR_ROPE) {
        const int half = p.d >> 1;
        const int i = i0 + rp_sel;
        const int ra = head * p.d + i;
        const float* bias = p.bias[sec];
        if (bias) {
            va = __fadd_rn(va, bias[ra]);
            vb = __fadd_rn(vb, bias[ra + half]);
        }
        const int seq = tok / p.n_tok, t = tok - seq * p.n_tok;
        const size_t pos = (size_t)p.n_past + t;
        const size_t kvw = (size_t)p.n_head_kv * p.d;
        if (sec == 2) {
            float* cv = p.cache_v + (size_t)seq * p.cache_bs + pos * kvw + ra;
            cv[0] = va;
            cv[half] = vb;
            return;
        }
        // separately rounded products and sums, as the reference's rope
        const float c = p.cos_tab[pos * half + i], s = p.sin_tab[pos * half + i];
        const float lo = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
        const float hi = __fadd_rn(__fmul_rn(va, s), __fmul_rn(vb, c));
        if (sec == 0) {
            float* qo = p.q_out + (size_t)tok * p.n_head * p.d + ra;
            qo[0] = lo;
            qo[half] = hi;
        } else {
            float* kt = p.cache_kt + (size_t)seq * p.cache_bs;
            kt[(size_t)ra * p.n_ctx + pos] = lo;
            kt[(size_t)(ra + half) * p.n_ctx + pos] = hi;
        }
    } else {
        // gate / (1 + exp(-gate)) * up
        const float sg = __fdiv_rn(va, __fadd_rn(1.0f, expf(-va)));
        p.out[(size_t)tok * p.n_pairs + i0 + rp_sel] = __fmul_rn(sg, vb);
    }
}

// Rows per warp (rw), k steps in flight per lane (unr) and k splits per row (ks) for an x
// chunk of mc rows, from a sweep of all three on B200 over the Qwen2.5 and Whisper shapes
// (one decode step's chain of launches in a CUDA graph). Four rows per warp (two pairs)
// won everywhere: each x value loaded then serves four rows. A matrix that gives 1.5 CTAs
// per SM with whole rows keeps them (unr = 2 when the grid is one wave at two CTAs per SM,
// so each lane has eight loads in flight); a smaller one splits its rows over 2, 4 or 8
// warps until it does, which also cuts the dependent steps of long rows (w_down: 18 steps
// of 512 bytes become 3 per warp). With 3-8 x rows the arithmetic per weight is larger and
// a warp takes four rows over the whole k.
struct Plan {
    int rw, unr, ks;
};

inline Plan plan(int mc, size_t rows, int pair, int sms) {
    if (mc > 2) return {4, 1, 1};
    const size_t rows_per_warp = pair ? 2 : 4;  // pairs or rows
    auto ctas = [&](int ks) { return (rows + (size_t)(WARPS / ks) * rows_per_warp - 1) / ((size_t)(WARPS / ks) * rows_per_warp); };
    const size_t want = (size_t)sms * 3 / 2;
    if (ctas(1) >= want) return {4, ctas(1) <= (size_t)(2 * sms) ? 2 : 1, 1};
    int ks = 2;
    while (ks < 8 && ctas(ks) < want) ks *= 2;
    return {4, 1, ks};
}

template <int MR, int UNR, int KS>
cudaError_t linear_cfg(dim3 grid, cudaStream_t st, const float* x, int mc, int k, const int8_t* wq, const float* ws,
                       const float* bias, int n, int mode, float* out) {
    return launch_chained(q8_linear_kernel<MR, 4, KS, UNR>, grid, dim3(32 * WARPS), st, x, mc, k, wq, ws, bias, n,
                          mode, out);
}

template <int MR>
cudaError_t linear_chunk(Plan pl, dim3 grid, cudaStream_t st, const float* x, int mc, int k, const int8_t* wq,
                         const float* ws, const float* bias, int n, int mode, float* out) {
    if constexpr (MR <= 2) {
        switch (pl.ks) {
            case 2: return linear_cfg<MR, 1, 2>(grid, st, x, mc, k, wq, ws, bias, n, mode, out);
            case 4: return linear_cfg<MR, 1, 4>(grid, st, x, mc, k, wq, ws, bias, n, mode, out);
            case 8: return linear_cfg<MR, 1, 8>(grid, st, x, mc, k, wq, ws, bias, n, mode, out);
            default:
                if (pl.unr == 2) return linear_cfg<MR, 2, 1>(grid, st, x, mc, k, wq, ws, bias, n, mode, out);
                return linear_cfg<MR, 1, 1>(grid, st, x, mc, k, wq, ws, bias, n, mode, out);
        }
    } else {
        return linear_cfg<MR, 1, 1>(grid, st, x, mc, k, wq, ws, bias, n, mode, out);
    }
}

template <int MR, int EPI>
cudaError_t pair_chunk(Plan pl, int rp, unsigned grid, cudaStream_t st, const PairParams& p) {
    const dim3 g(grid), b(32 * WARPS);
    if (rp == 1) return launch_chained(q8_pair_kernel<MR, 1, 1, 1, EPI>, g, b, st, p);
    if constexpr (MR <= 2) {
        switch (pl.ks) {
            case 2: return launch_chained(q8_pair_kernel<MR, 2, 2, 1, EPI>, g, b, st, p);
            case 4: return launch_chained(q8_pair_kernel<MR, 2, 4, 1, EPI>, g, b, st, p);
            case 8: return launch_chained(q8_pair_kernel<MR, 2, 8, 1, EPI>, g, b, st, p);
            default:
                if (pl.unr == 2) return launch_chained(q8_pair_kernel<MR, 2, 1, 2, EPI>, g, b, st, p);
                break;
        }
    }
    return launch_chained(q8_pair_kernel<MR, 2, 1, 1, EPI>, g, b, st, p);
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

static int sm_count_current() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

int q8_linear_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias,
                     size_t n, int mode, float* out, cudaStream_t st) {
    if (m == 0 || n == 0) return 0;
    const int sms = sm_count_current();
    const int ik = (int)k, in = (int)n;
    // many rows of x: the register-tiled product, the weights read once per 32 rows
    if (m >= 16) return q8_gemm_launch(x, m, k, wq, ws, bias, n, mode, out, sms, st);
    for (size_t m0 = 0; m0 < m; m0 += 8) {
        const int mc = (int)std::min<size_t>(8, m - m0);
        const float* xc = x + m0 * k;
        float* oc = out + m0 * n;
        const q8::Plan pl = q8::plan(mc, n, 0, sms);
        const size_t rows_per_cta = (size_t)(q8::WARPS / pl.ks) * pl.rw;
        const dim3 grid((unsigned)((n + rows_per_cta - 1) / rows_per_cta));
        cudaError_t e;
        if (mc == 1) e = q8::linear_chunk<1>(pl, grid, st, xc, mc, ik, wq, ws, bias, in, mode, oc);
        else if (mc == 2) e = q8::linear_chunk<2>(pl, grid, st, xc, mc, ik, wq, ws, bias, in, mode, oc);
        else if (mc <= 4) e = q8::linear_chunk<4>(pl, grid, st, xc, mc, ik, wq, ws, bias, in, mode, oc);
        else e = q8::linear_chunk<8>(pl, grid, st, xc, mc, ik, wq, ws, bias, in, mode, oc);
        if (e != cudaSuccess) return -1;
    }
    return 0;
}

int q8_pair_launch(const PairParams& p0, int epi, cudaStream_t st) {
    if (p0.m == 0 || p0.n_pairs == 0) return 0;
    const int sms = sm_count_current();
    // many rows of x: the pairs on the register-tiled product
    if (epi == PAIR_ROPE && p0.m >= 16) return q8_gemm_rope_launch(p0, sms, st);
    if (epi == PAIR_SILU && p0.m >= 16)
        return q8_gemm_silu_launch(p0.x, (size_t)p0.m, (size_t)p0.k, p0.wq[0], p0.ws[0], p0.bias[0], p0.wq[1], p0.ws[1],
                                   p0.bias[1], (size_t)p0.n_pairs, p0.out + (size_t)p0.m0 * p0.n_pairs, sms, st);
    PairParams p = p0;
    for (int m0 = 0; m0 < p0.m; m0 += 8) {
        const int mc = std::min(8, p0.m - m0);
        p.x = p0.x + (size_t)m0 * p0.k;
        p.m = mc;
        p.m0 = p0.m0 + m0;
        q8::Plan pl = q8::plan(mc, (size_t)p0.n_pairs, 1, sms);
        int rp = pl.rw / 2;
        if (epi == PAIR_ROPE && (p0.d / 2) % rp) rp = 1;  // the pairs of a warp stay in one head
        if (rp == 1) pl.ks = 1;
        const size_t pairs_per_cta = (size_t)(q8::WARPS / pl.ks) * rp;
        const unsigned grid = (unsigned)((p0.n_pairs + pairs_per_cta - 1) / pairs_per_cta);
        cudaError_t e;
        if (epi == PAIR_ROPE) {
            if (mc == 1) e = q8::pair_chunk<1, PAIR_ROPE>(pl, rp, grid, st, p);
            else if (mc == 2) e = q8::pair_chunk<2, PAIR_ROPE>(pl, rp, grid, st, p);
            else if (mc <= 4) e = q8::pair_chunk<4, PAIR_ROPE>(pl, rp, grid, st, p);
            else e = q8::pair_chunk<8, PAIR_ROPE>(pl, rp, grid, st, p);
        } else {
            if (mc == 1) e = q8::pair_chunk<1, PAIR_SILU>(pl, rp, grid, st, p);
            else if (mc == 2) e = q8::pair_chunk<2, PAIR_SILU>(pl, rp, grid, st, p);
            else if (mc <= 4) e = q8::pair_chunk<4, PAIR_SILU>(pl, rp, grid, st, p);
            else e = q8::pair_chunk<8, PAIR_SILU>(pl, rp, grid, st, p);
        }
        if (e != cudaSuccess) return -1;
    }
    return 0;
}

}  // namespace zwg
