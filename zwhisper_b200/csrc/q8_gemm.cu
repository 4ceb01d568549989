// Q8 products for 16 or more rows of activations (ops.linear with Q8 weights, src/ops.zig:
// 280-306 -> gemm.ntBlockQ, src/gemm.zig:268-351): out[i][j] = sum over k of x[i][k] * w[j][k]
// with w = q * scale (the dequantized weight of Q8.row, src/gemm.zig:256-263), + bias[j], then
// the epilogue of q8_linear_kernel (store, add into out, or tanh GELU).
//
// At 16-64 rows (a decoder step over 32 windows, an LLM step over 64 sequences, the 1500 rows
// of setAudio) the weight bytes are read once per tile instead of once per 8 rows, and the
// work is f32 FMA: a register-tiled product. Shapes with at least 64 tiles of 32 or 64 rows
// x 128 columns take those (q8g below: 8 x 8 outputs per thread, the dequantized weights
// staged, four 16-byte shared loads per 64 FMAs); the others take 32 x 64 tiles (q8s: 4 x 4
// outputs per thread, the block's dots formed unscaled and added times the block's scales).
// Per 32-wide k block a CTA stages x and the weights k-major in shared memory,
// double-buffered through registers.
//
// Split-K without a workspace: when the tiles alone would leave SMs idle, a cluster of ks
// CTAs (1 x 1 x ks) takes one tile, each CTA a contiguous range of k blocks; the CTAs then
// leave their partial tiles in shared memory and each reduces its share of the rows over the
// cluster's CTAs in rank order through distributed shared memory (deterministic), and writes
// the epilogue. The kernel has no spin waits: only block and cluster barriers, which every
// thread reaches.
//
// Fused modes on the same tiles (the pair kernels of q8.cu for many rows, and one more): the
// SiLU pair (gate and up, src/llm.zig:206-208) and the RoPE pair (q/k/v + bias + rotation +
// cache append, src/llm.zig:179-190), a thread owning the same columns of both row sets; and
// the Whisper decoder's q/k/v as one product whose epilogue appends k and v to the caches
// (src/decoder.zig:180-183).
//
// Launched as a programmatic dependent (chain.cuh): the weight rows of the CTA's k range are
// prefetched into L2 before the wait for the kernel that wrote x.
#include <type_traits>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "chain.cuh"
#include "common.cuh"
#include "kernels.h"

namespace zwg {

namespace q8g {

constexpr int BN = 128, BK = 32, MAX_KS = 8;

template <int BM>
struct Smem {
    union {
        struct {
            float xs[2][BK][BM];  // x block, k-major
            float ws[2][BK][BN];  // dequantized weights of the block, k-major
        } s;
        float red[BM][BN];        // this CTA's partial tile (split-K), after the k loop
    };
};

__device__ __forceinline__ float gelu_tanh(float x) {
    const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(u)));
}

__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_cluster(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

__device__ __forceinline__ void finish_pair(float* out, const float* bias_g, const float* bias_u, int n, int row,
                                            int col, float g, float u) {
    if (bias_g) g = __fadd_rn(g, __ldg(bias_g + col));
    if (bias_u) u = __fadd_rn(u, __ldg(bias_u + col));
    out[(size_t)row * n + col] = silu_mul(g, u);
}

template <int MODE>
__device__ __forceinline__ void finish(float* out, const float* bias, int n, int row, int col, float v) {
    if (bias) v = __fadd_rn(v, __ldg(bias + col));
    float* o = out + (size_t)row * n + col;
    if (MODE == LIN_ADD) v = __fadd_rn(__ldcg(o), v);
    else if (MODE == LIN_GELU) v = gelu_tanh(v);
    *o = v;
}

// Pair modes: two output rows that one epilogue needs together share a thread.
//   PE_SILU: row j of the gate matrix (the args' wq / ws / bias) and of pp.wq[1] (up).
//   PE_ROPE: rows i and i + d/2 of one head of wq, wk or wv (pp.wq[0..2]); the epilogue of
//            q8_pair_kernel's PAIR_ROPE (bias, rotation, q out, K^T scatter, V copy).
// And one column mode that is not a pair:
//   PE_QKV:  the Whisper decoder's self-attention projections as one product over the 3 d
//            columns of wq, wk and wv (pp.wq[0..2], d = pp.d rows each, biases pp.bias[]):
//            q to pp.q_out, k and v appended to the decoder caches (pp.cache_kt / cache_v,
//            window w at w * cache_bs, position n_past + t, row stride d).
enum { PE_NONE = 0, PE_SILU = 1, PE_ROPE = 2, PE_QKV = 3 };

// Matrix (0 q, 1 k, 2 v) and row of pair pc's first (second: + d/2) row in PE_ROPE.
__device__ __forceinline__ void rope_row(const PairParams& p, int pc, bool second, int& sec, int& row) {
    const int half = p.d >> 1;
    const int hh = pc / half, i0 = pc - hh * half;
    sec = hh < p.n_head ? 0 : hh < p.n_head + p.n_head_kv ? 1 : 2;
    const int head = sec == 0 ? hh : sec == 1 ? hh - p.n_head : hh - p.n_head - p.n_head_kv;
    row = head * p.d + i0 + (second ? half : 0);
}

// Loader row wj of a tile of TBN columns starting at output n0: the matrix, its scales, the
// row, and whether the row exists (outputs past n are not stored).
template <int PE, int TBN>
__device__ __forceinline__ void tile_row(int wj, int n0, int n, const int8_t* wq, const float* ws,
                                         const PairParams& pp, const int8_t*& base, const float*& sbase, int& row,
                                         bool& ok) {
    if (PE == PE_NONE) {
        row = n0 + wj;
        ok = row < n;
        base = wq;
        sbase = ws;
        return;
    }
    if (PE == PE_QKV) {
        const int vc = n0 + wj;
        ok = vc < n;
        const int sel = ok ? vc / pp.d : 0;
        row = ok ? vc - sel * pp.d : 0;
        base = pp.wq[sel];
        sbase = pp.ws[sel];
        return;
    }
    const bool second = wj >= TBN / 2;
    const int pc = n0 + (second ? wj - TBN / 2 : wj);
    ok = pc < n;
    if (PE == PE_SILU) {
        row = pc;
        base = second ? pp.wq[1] : wq;
        sbase = second ? pp.ws[1] : ws;
    } else {
        int sec;
        rope_row(pp, ok ? pc : 0, second, sec, row);
        base = pp.wq[sec];
        sbase = pp.ws[sec];
    }
}

// PAIR_ROPE's epilogue for x row r of the call and pair pc (q8_pair_kernel, q8.cu).
__device__ __forceinline__ void finish_rope(const PairParams& p, int r, int pc, float va, float vb) {
    int sec, ra;
    rope_row(p, pc, false, sec, ra);
    const int half = p.d >> 1, i = ra % p.d;
    const float* bias = p.bias[sec];
    if (bias) {
        va = __fadd_rn(va, __ldg(bias + ra));
        vb = __fadd_rn(vb, __ldg(bias + ra + half));
    }
    const int tok = p.m0 + r;
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
}

// PE_QKV's epilogue for x row r of the call (window r / n_tok, token r % n_tok) and column vc.
__device__ __forceinline__ void finish_qkv(const PairParams& p, int r, int vc, float v) {
    const int sel = vc / p.d, col = vc - sel * p.d;
    if (p.bias[sel]) v = __fadd_rn(v, __ldg(p.bias[sel] + col));
    if (sel == 0) {
        p.q_out[(size_t)r * p.d + col] = v;
        return;
    }
    const int seq = r / p.n_tok, t = r - seq * p.n_tok;
    float* cache = sel == 1 ? p.cache_kt : p.cache_v;
    cache[(size_t)seq * p.cache_bs + ((size_t)p.n_past + t) * p.d + col] = v;
}

// The epilogue of one output column (not a pair).
template <int MODE, int PE>
__device__ __forceinline__ void finish_one(float* out, const float* bias, const PairParams& pp, int n, int row, int col,
                                           float v) {
    if (PE == PE_QKV) finish_qkv(pp, row, col, v);
    else finish<MODE>(out, bias, n, row, col, v);
}

// The epilogue of one output pair.
template <int PE>
__device__ __forceinline__ void finish_two(float* out, const float* bias, const PairParams& pp, int n, int row, int col,
                                           float a, float b) {
    if (PE == PE_SILU) finish_pair(out, bias, pp.bias[1], n, row, col, a, b);
    else finish_rope(pp, row, col, a, b);
}

// Tile column of output j (0..7) of thread tx: columns tx*4..+3 of each 64-column half (for
// the SiLU pair the gate and the up half).
__device__ __forceinline__ int tile_col(int tx, int j) { return (j < 4 ? 0 : BN / 2) + tx * 4 + (j & 3); }

// MODE: LIN_STORE / LIN_ADD / LIN_GELU (PE_NONE); PE: a pair mode (n = the number of pairs);
// BM: rows of x per tile (32 or 64), threads = BM / 8 * 16.
template <int MODE, int PE, int BM>
__global__ void __launch_bounds__(BM * 2) q8_gemm_kernel(const float* x, int m, int k, const int8_t* __restrict__ wq,
                                                        const float* __restrict__ ws, const float* __restrict__ bias,
                                                        int n, float* out, int ks, PairParams pp) {
    constexpr bool PAIR = PE == PE_SILU || PE == PE_ROPE;
    constexpr int THREADS = BM * 2;
    constexpr int XL = BM * BK / 4 / THREADS;    // x float4 per thread per block (4)
    constexpr int WL = BN * BK / 16 / THREADS;   // weight 16-byte pieces per thread per block
    __shared__ __align__(16) Smem<BM> sm;
    const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
    // a tile's first output column: 128 columns, or 64 gate / up pairs
    const int n0 = blockIdx.x * (PAIR ? BN / 2 : BN), m0 = blockIdx.y * BM, kz = blockIdx.z;
    const int nb = k / BK;
    const int b_beg = (int)((long long)kz * nb / ks), b_end = (int)((long long)(kz + 1) * nb / ks);
    // weight loader rows: piece t + i * THREADS is row (.) >> 1, sixteen k at ((.) & 1) * 16
    const int8_t* wrow[WL];
    const float* wsc[WL];
    bool wok[WL];
#pragma unroll
    for (int i = 0; i < WL; i++) {
        const int wj = (t + i * THREADS) >> 1;
        const int8_t* base;
        const float* sbase;
        int wn;
        tile_row<PE, BN>(wj, n0, n, wq, ws, pp, base, sbase, wn, wok[i]);
        wrow[i] = base + (size_t)(wok[i] ? wn : 0) * k;
        wsc[i] = sbase + (size_t)(wok[i] ? wn : 0) * nb;
        // the weights are constants: their rows of this k range go to L2 before the wait
        if (wok[i] && ((t + i * THREADS) & 1) == 0)
            for (int off = b_beg * BK; off < b_end * BK; off += 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(wrow[i] + off));
    }
    chain_release();
    const int z = chain_wait();
    x += z;
    out += z;

    float4 xr[XL];
    uint4 qr[WL];
    float sr[WL];
    auto load = [&](int kb) {
#pragma unroll
        for (int i = 0; i < XL; i++) {
            const int idx = t + i * THREADS, row = m0 + (idx >> 3), kq = (idx & 7) * 4;
            xr[i] = row < m ? *reinterpret_cast<const float4*>(x + (size_t)row * k + kb * BK + kq)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < WL; i++) {
            const int h = (t + i * THREADS) & 1;
            qr[i] = wok[i] ? __ldg(reinterpret_cast<const uint4*>(wrow[i] + kb * BK + h * 16)) : make_uint4(0, 0, 0, 0);
            sr[i] = wok[i] ? __ldg(wsc[i] + kb) : 0.f;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < XL; i++) {
            const int idx = t + i * THREADS, row = idx >> 3, kq = (idx & 7) * 4;
            sm.s.xs[buf][kq][row] = xr[i].x;
            sm.s.xs[buf][kq + 1][row] = xr[i].y;
            sm.s.xs[buf][kq + 2][row] = xr[i].z;
            sm.s.xs[buf][kq + 3][row] = xr[i].w;
        }
#pragma unroll
        for (int i = 0; i < WL; i++) {
            const int idx = t + i * THREADS, wj = idx >> 1, h = idx & 1;
            const uint32_t words[4] = {qr[i].x, qr[i].y, qr[i].z, qr[i].w};
#pragma unroll
            for (int wdx = 0; wdx < 4; wdx++)
#pragma unroll
                for (int byte = 0; byte < 4; byte++)
                    sm.s.ws[buf][h * 16 + wdx * 4 + byte][wj] =
                        __fmul_rn((float)(int8_t)(words[wdx] >> (8 * byte)), sr[i]);
        }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;
    if (b_beg < b_end) {
        load(b_beg);
        store(0);
    }
    __syncthreads();
    for (int kb = b_beg; kb < b_end; kb++) {
        const int buf = (kb - b_beg) & 1;
        if (kb + 1 < b_end) load(kb + 1);
#pragma unroll 4
        for (int kk = 0; kk < BK; kk++) {
            const float4 a0 = *reinterpret_cast<const float4*>(&sm.s.xs[buf][kk][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&sm.s.xs[buf][kk][ty * 8 + 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&sm.s.ws[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&sm.s.ws[buf][kk][BN / 2 + tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (kb + 1 < b_end) store(buf ^ 1);
        __syncthreads();
    }

    if (ks == 1) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int row = m0 + ty * 8 + i;
            if (row >= m) continue;
            if (PAIR) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int col = n0 + tx * 4 + j;
                    if (col < n) finish_two<PE>(out, bias, pp, n, row, col, acc[i][j], acc[i][4 + j]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int col = n0 + tile_col(tx, j);
                    if (col < n) finish_one<MODE, PE>(out, bias, pp, n, row, col, acc[i][j]);
                }
            }
        }
        return;
    }
    // split-K: partial tiles in shared memory (over the staging buffers, all reads of which
    // ended at the loop's last barrier), each CTA reduces BM / ks rows over the cluster
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) sm.red[ty * 8 + i][tile_col(tx, j)] = acc[i][j];
    cluster_sync_all();
    const int rows = BM / ks, r0 = kz * rows;
    constexpr int OUTS = PAIR ? BN / 2 : BN;  // outputs per tile row
    // every rank's values of 16 / ks outputs are loaded before the first add, so a batch
    // costs one round trip through the cluster instead of one per output (ks is 2, 4 or 8;
    // the sums keep rank order)
    auto reduce = [&](auto ks_c) {
        constexpr int KS = decltype(ks_c)::value;
        constexpr int EB = 16 / KS;  // outputs per batch
        const int total = rows * OUTS;
        for (int e0 = t; e0 < total; e0 += EB * THREADS) {
            float pv[EB][KS], pu[EB][KS];
#pragma unroll
            for (int b = 0; b < EB; b++) {
                // outputs past the share load one of it (in bounds) and are not used
                const int e = min(e0 + b * THREADS, total - 1);
                const int rr = r0 + e / OUTS, cc = e % OUTS;
#pragma unroll
                for (int q = 0; q < KS; q++) {
                    pv[b][q] = ld_cluster(cluster_addr(&sm.red[rr][cc], (uint32_t)q));
                    pu[b][q] = PAIR ? ld_cluster(cluster_addr(&sm.red[rr][BN / 2 + cc], (uint32_t)q)) : 0.f;
                }
            }
#pragma unroll
            for (int b = 0; b < EB; b++) {
                const int e = e0 + b * THREADS;
                if (e >= total) break;
                const int rr = r0 + e / OUTS, cc = e % OUTS;
                const int row = m0 + rr, col = n0 + cc;
                float v = 0.f, u = 0.f;
#pragma unroll
                for (int q = 0; q < KS; q++) {
                    v = __fadd_rn(v, pv[b][q]);
                    if (PAIR) u = __fadd_rn(u, pu[b][q]);
                }
                if (row < m && col < n) {
                    if (PAIR) finish_two<PE>(out, bias, pp, n, row, col, v, u);
                    else finish_one<MODE, PE>(out, bias, pp, n, row, col, v);
                }
            }
        }
    };
    if (ks == 2) reduce(std::integral_constant<int, 2>{});
    else if (ks == 4) reduce(std::integral_constant<int, 4>{});
    else reduce(std::integral_constant<int, 8>{});
    // no CTA leaves while another may still read its partial tile
    cluster_sync_all();
}

}  // namespace q8g

// The small-tile kernel for shapes that give few 64 x 128 tiles (a decoder step's 512 x 512
// projections, an LLM layer's output and down projections at 64 rows): tiles of 32 x 64, 4 x
// 4 outputs per thread, the block's dots formed unscaled and added times the block's scales,
// and more k splits.
namespace q8s {

constexpr int BM = 32, BN = 64, BK = 32, THREADS = 128, MAX_KS = 8;

struct Smem {
    float xs[2][BK][BM];  // x block, k-major
    float wq[2][BK][BN];  // int8 weights of the block as floats, k-major
    float sc[2][BN];      // the block's scale of each column
    float red[BM][BN];    // this CTA's partial tile (split-K)
};

using q8g::cluster_addr;
using q8g::cluster_sync_all;
using q8g::finish;
using q8g::finish_one;
using q8g::finish_two;
using q8g::ld_cluster;
using q8g::PE_NONE;
using q8g::PE_ROPE;
using q8g::PE_SILU;
using q8g::tile_row;

template <bool PAIR>
__device__ __forceinline__ int tile_col(int tx, int j) {
    return PAIR ? (j < 2 ? tx * 2 + j : BN / 2 + tx * 2 + (j - 2)) : tx * 4 + j;
}

// MODE: LIN_STORE / LIN_ADD / LIN_GELU (PE_NONE); PE: a pair mode.
template <int MODE, int PE>
__global__ void __launch_bounds__(THREADS) q8_gemm_kernel(const float* x, int m, int k, const int8_t* __restrict__ wq,
                                                          const float* __restrict__ ws, const float* __restrict__ bias,
                                                          int n, float* out, int ks, PairParams pp) {
    constexpr bool PAIR = PE == PE_SILU || PE == PE_ROPE;
    __shared__ __align__(16) Smem sm;
    const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
    // a tile's first output column: 64 columns, or 32 gate / up pairs
    const int n0 = blockIdx.x * (PAIR ? BN / 2 : BN), m0 = blockIdx.y * BM, kz = blockIdx.z;
    const int nb = k / BK;
    const int b_beg = (int)((long long)kz * nb / ks), b_end = (int)((long long)(kz + 1) * nb / ks);
    // loader roles: x rows (t >> 3) and (t >> 3) + 16, four k at (t & 7) * 4; weight row t >> 1,
    // sixteen k at (t & 1) * 16
    const int xrow = t >> 3, xk = (t & 7) * 4, wj = t >> 1, wh = t & 1;
    const int8_t* base;
    const float* sbase;
    int wn;
    bool wrow_ok;
    tile_row<PE, BN>(wj, n0, n, wq, ws, pp, base, sbase, wn, wrow_ok);
    const int8_t* wrow = base + (size_t)(wrow_ok ? wn : 0) * k;
    const float* wsc = sbase + (size_t)(wrow_ok ? wn : 0) * nb;
    // the weights are constants: their rows of this k range go to L2 before the wait
    if (wrow_ok)
        for (int off = b_beg * BK + wh * 128; off < b_end * BK; off += 256)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(wrow + off));
    chain_release();
    const int z = chain_wait();
    x += z;
    out += z;

    float4 xr[2];
    uint4 qr;
    float sr = 0.f;
    auto load = [&](int kb) {
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int row = m0 + xrow + 16 * i;
            xr[i] = row < m ? *reinterpret_cast<const float4*>(x + (size_t)row * k + kb * BK + xk)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        qr = wrow_ok ? __ldg(reinterpret_cast<const uint4*>(wrow + kb * BK + wh * 16)) : make_uint4(0, 0, 0, 0);
        if (wh == 0) sr = wrow_ok ? __ldg(wsc + kb) : 0.f;
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int row = xrow + 16 * i;
            sm.xs[buf][xk][row] = xr[i].x;
            sm.xs[buf][xk + 1][row] = xr[i].y;
            sm.xs[buf][xk + 2][row] = xr[i].z;
            sm.xs[buf][xk + 3][row] = xr[i].w;
        }
        const uint32_t words[4] = {qr.x, qr.y, qr.z, qr.w};
#pragma unroll
        for (int wdx = 0; wdx < 4; wdx++)
#pragma unroll
            for (int byte = 0; byte < 4; byte++)
                sm.wq[buf][wh * 16 + wdx * 4 + byte][wj] = (float)(int8_t)(words[wdx] >> (8 * byte));
        if (wh == 0) sm.sc[buf][wj] = sr;
    };

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
    if (b_beg < b_end) {
        load(b_beg);
        store(0);
    }
    __syncthreads();
    for (int kb = b_beg; kb < b_end; kb++) {
        const int buf = (kb - b_beg) & 1;
        if (kb + 1 < b_end) load(kb + 1);
        float p[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) p[i][j] = 0.f;
#pragma unroll 8
        for (int kk = 0; kk < BK; kk++) {
            const float4 a = *reinterpret_cast<const float4*>(&sm.xs[buf][kk][ty * 4]);
            float bv[4];
            if (PAIR) {
                const float2 b0 = *reinterpret_cast<const float2*>(&sm.wq[buf][kk][tx * 2]);
                const float2 b1 = *reinterpret_cast<const float2*>(&sm.wq[buf][kk][BN / 2 + tx * 2]);
                bv[0] = b0.x, bv[1] = b0.y, bv[2] = b1.x, bv[3] = b1.y;
            } else {
                const float4 b = *reinterpret_cast<const float4*>(&sm.wq[buf][kk][tx * 4]);
                bv[0] = b.x, bv[1] = b.y, bv[2] = b.z, bv[3] = b.w;
            }
            const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) p[i][j] = fmaf(av[i], bv[j], p[i][j]);
        }
        float sv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) sv[j] = sm.sc[buf][tile_col<PAIR>(tx, j)];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = fmaf(p[i][j], sv[j], acc[i][j]);
        if (kb + 1 < b_end) store(buf ^ 1);
        __syncthreads();
    }

    if (ks == 1) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int row = m0 + ty * 4 + i;
            if (row >= m) continue;
            if (PAIR) {
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int col = n0 + tx * 2 + j;
                    if (col < n) finish_two<PE>(out, bias, pp, n, row, col, acc[i][j], acc[i][2 + j]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int col = n0 + tx * 4 + j;
                    if (col < n) finish_one<MODE, PE>(out, bias, pp, n, row, col, acc[i][j]);
                }
            }
        }
        return;
    }
    // split-K: partial tiles in shared memory, each CTA reduces BM / ks rows over the cluster
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) sm.red[ty * 4 + i][tile_col<PAIR>(tx, j)] = acc[i][j];
    cluster_sync_all();
    const int rows = BM / ks, r0 = kz * rows;
    constexpr int OUTS = PAIR ? BN / 2 : BN;  // outputs per tile row
    // every rank's values of 16 / ks outputs are loaded before the first add, so a batch
    // costs one round trip through the cluster instead of one per output (ks is 2, 4 or 8;
    // the sums keep rank order)
    auto reduce = [&](auto ks_c) {
        constexpr int KS = decltype(ks_c)::value;
        constexpr int EB = 16 / KS;  // outputs per batch
        const int total = rows * OUTS;
        for (int e0 = t; e0 < total; e0 += EB * THREADS) {
            float pv[EB][KS], pu[EB][KS];
#pragma unroll
            for (int b = 0; b < EB; b++) {
                // outputs past the share load one of it (in bounds) and are not used
                const int e = min(e0 + b * THREADS, total - 1);
                const int rr = r0 + e / OUTS, cc = e % OUTS;
#pragma unroll
                for (int q = 0; q < KS; q++) {
                    pv[b][q] = ld_cluster(cluster_addr(&sm.red[rr][cc], (uint32_t)q));
                    pu[b][q] = PAIR ? ld_cluster(cluster_addr(&sm.red[rr][BN / 2 + cc], (uint32_t)q)) : 0.f;
                }
            }
#pragma unroll
            for (int b = 0; b < EB; b++) {
                const int e = e0 + b * THREADS;
                if (e >= total) break;
                const int rr = r0 + e / OUTS, cc = e % OUTS;
                const int row = m0 + rr, col = n0 + cc;
                float v = 0.f, u = 0.f;
#pragma unroll
                for (int q = 0; q < KS; q++) {
                    v = __fadd_rn(v, pv[b][q]);
                    if (PAIR) u = __fadd_rn(u, pu[b][q]);
                }
                if (row < m && col < n) {
                    if (PAIR) finish_two<PE>(out, bias, pp, n, row, col, v, u);
                    else finish_one<MODE, PE>(out, bias, pp, n, row, col, v);
                }
            }
        }
    };
    if (ks == 2) reduce(std::integral_constant<int, 2>{});
    else if (ks == 4) reduce(std::integral_constant<int, 4>{});
    else reduce(std::integral_constant<int, 8>{});
    // no CTA leaves while another may still read its partial tile
    cluster_sync_all();
}

}  // namespace q8s

namespace {

// k splits (powers of two, at most 8, at least two k blocks each) while the tiles alone
// would give fewer than two CTAs per SM
int k_splits(size_t tiles, size_t nb, int sm_count) {
    int ks = 1;
    while (ks < q8g::MAX_KS && tiles * ks < 2 * (size_t)std::max(1, sm_count) && nb / (2 * ks) >= 2) ks *= 2;
    return ks;
}

int launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias, size_t n,
           int mode, int pe, const PairParams& pp, float* out, int sm_count, cudaStream_t st) {
    using namespace q8g;
    const bool pair = pe == PE_SILU || pe == PE_ROPE;
    if (m == 0 || n == 0) return 0;
    if (k == 0 || k % q8g::BK || ((uintptr_t)x & 15) || ((uintptr_t)wq & 15)) return -1;
    for (int i = 0; i < (pe == PE_ROPE || pe == PE_QKV ? 3 : pe == PE_SILU ? 2 : 0); i++)
        if (!pp.wq[i] || ((uintptr_t)pp.wq[i] & 15)) return -1;
    if (m > (1u << 30) || n > (1u << 30) || k > (1u << 30)) return -1;
    const size_t nb = k / q8g::BK;
    // the large tiles (32 or 64 rows x 128 columns) when the shape gives at least 64 of them
    // (measured on B200: the logits, an LLM layer's gate/up pair), else the small ones
    const int bm = m <= 32 ? 32 : 64;
    const size_t big_n = (n + (pair ? q8g::BN / 2 : q8g::BN) - 1) / (pair ? q8g::BN / 2 : q8g::BN);
    const size_t big_m = (m + bm - 1) / bm;
    const bool big = big_n * big_m >= 64;
    const size_t small_n = (n + (pair ? q8s::BN / 2 : q8s::BN) - 1) / (pair ? q8s::BN / 2 : q8s::BN);
    const size_t small_m = (m + q8s::BM - 1) / q8s::BM;
    const size_t tiles_n = big ? big_n : small_n, tiles_m = big ? big_m : small_m;
    if (tiles_m > 65535 || tiles_n > 0x7fffffff) return -1;
    const int ks = k_splits(tiles_n * tiles_m, nb, sm_count);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)ks);
    cfg.blockDim = dim3((unsigned)(big ? 2 * bm : q8s::THREADS));
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = (unsigned)ks;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int im = (int)m, ik = (int)k, in = (int)n;
    auto go = [&](auto kern) {
        return cudaLaunchKernelEx(&cfg, kern, x, im, ik, wq, ws, bias, in, out, ks, pp) == cudaSuccess ? 0 : -1;
    };
    using q8g::q8_gemm_kernel;
    if (!big) {
        if (pe == PE_SILU) return go(q8s::q8_gemm_kernel<LIN_STORE, PE_SILU>);
        if (pe == PE_ROPE) return go(q8s::q8_gemm_kernel<LIN_STORE, PE_ROPE>);
        if (pe == PE_QKV) return go(q8s::q8_gemm_kernel<LIN_STORE, PE_QKV>);
        if (mode == LIN_ADD) return go(q8s::q8_gemm_kernel<LIN_ADD, PE_NONE>);
        if (mode == LIN_GELU) return go(q8s::q8_gemm_kernel<LIN_GELU, PE_NONE>);
        return go(q8s::q8_gemm_kernel<LIN_STORE, PE_NONE>);
    }
    if (bm == 32) {
        if (pe == PE_SILU) return go(q8_gemm_kernel<LIN_STORE, PE_SILU, 32>);
        if (pe == PE_ROPE) return go(q8_gemm_kernel<LIN_STORE, PE_ROPE, 32>);
        if (pe == PE_QKV) return go(q8_gemm_kernel<LIN_STORE, PE_QKV, 32>);
        if (mode == LIN_ADD) return go(q8_gemm_kernel<LIN_ADD, PE_NONE, 32>);
        if (mode == LIN_GELU) return go(q8_gemm_kernel<LIN_GELU, PE_NONE, 32>);
        return go(q8_gemm_kernel<LIN_STORE, PE_NONE, 32>);
    }
    if (pe == PE_SILU) return go(q8_gemm_kernel<LIN_STORE, PE_SILU, 64>);
    if (pe == PE_ROPE) return go(q8_gemm_kernel<LIN_STORE, PE_ROPE, 64>);
    if (pe == PE_QKV) return go(q8_gemm_kernel<LIN_STORE, PE_QKV, 64>);
    if (mode == LIN_ADD) return go(q8_gemm_kernel<LIN_ADD, PE_NONE, 64>);
    if (mode == LIN_GELU) return go(q8_gemm_kernel<LIN_GELU, PE_NONE, 64>);
    return go(q8_gemm_kernel<LIN_STORE, PE_NONE, 64>);
}

}  // namespace

// out[m][n] (+)= x[m][k] . W^T (meant for m >= 16), k a multiple of 32; mode as
// q8_linear_launch. Returns -1 on a bad argument or a launch failure.
int q8_gemm_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias, size_t n,
                   int mode, float* out, int sm_count, cudaStream_t st) {
    if (m > 0 && n > 0) {
        const int r = q8_tc_launch(x, m, k, wq, ws, bias, n, mode, nullptr, nullptr, nullptr, out, sm_count, st);
        if (r != 1) return r;
    }
    const PairParams none{};
    return launch(x, m, k, wq, ws, bias, n, mode, q8g::PE_NONE, none, out, sm_count, st);
}

// out[m][n_ff] = silu(x . Wg^T + bg) * (x . Wu^T + bu), the SiLU pair of q8_pair_launch.
int q8_gemm_silu_launch(const float* x, size_t m, size_t k, const int8_t* wg, const float* sg, const float* bg,
                        const int8_t* wu, const float* su, const float* bu, size_t n_ff, float* out, int sm_count,
                        cudaStream_t st) {
    if (m > 0 && n_ff > 0 && wu) {
        const int r = q8_tc_launch(x, m, k, wg, sg, bg, n_ff, LIN_STORE, wu, su, bu, out, sm_count, st);
        if (r != 1) return r;
    }
    PairParams pp{};
    pp.wq[0] = wg;
    pp.ws[0] = sg;
    pp.bias[0] = bg;
    pp.wq[1] = wu;
    pp.ws[1] = su;
    pp.bias[1] = bu;
    return launch(x, m, k, wg, sg, bg, n_ff, LIN_STORE, q8g::PE_SILU, pp, out, sm_count, st);
}

// The Whisper decoder's q/k/v projections in one product (PE_QKV): p.x [m][p.k], p.wq/ws/bias
// [3], p.d = n_state, q to p.q_out, k / v rows appended to p.cache_kt / p.cache_v.
int q8_gemm_qkv_launch(const PairParams& p, int sm_count, cudaStream_t st) {
    if (p.m > 0 && p.d > 0) {
        const int r = q8_tc_qkv_launch(p, sm_count, st);
        if (r != 1) return r;
    }
    return launch(p.x, (size_t)p.m, (size_t)p.k, p.wq[0], p.ws[0], nullptr, (size_t)3 * p.d, LIN_STORE, q8g::PE_QKV,
                  p, nullptr, sm_count, st);
}

// The RoPE pair of q8_pair_launch (q/k/v + bias + RoPE + K^T / V append) on the tiles.
int q8_gemm_rope_launch(const PairParams& p, int sm_count, cudaStream_t st) {
    if (p.m > 0 && p.n_pairs > 0) {
        const int r = q8_tc_rope_launch(p, sm_count, st);
        if (r != 1) return r;
    }
    return launch(p.x, (size_t)p.m, (size_t)p.k, p.wq[0], p.ws[0], nullptr, (size_t)p.n_pairs, LIN_STORE, q8g::PE_ROPE,
                  p, nullptr, sm_count, st);
}

}  // namespace zwg
