// Q8 products for 16 or more rows of activations (ops.linear with Q8 weights, src/ops.zig:
// 280-306 -> gemm.ntBlockQ, src/gemm.zig:268-351): out[i][j] = sum over the k/32 blocks of
// scale[j][b] * (sum over the block of x[i][k] * q[j][k]), + bias[j], then the epilogue of
// q8_linear_kernel (store, add into out, or tanh GELU).
//
// At 16-64 rows (a decoder step over 32 windows, an LLM step over 64 sequences, the 1500 rows
// of setAudio) the weight bytes are read once per tile instead of once per 8 rows, and the
// work is f32 FMA: a register-tiled product, CTA tile 32 rows x 64 columns, 128 threads with
// 4 x 4 outputs each. Per 32-wide k block the CTA stages x (k-major) and the int8 weights as
// exact small floats (k-major) in shared memory, double-buffered through registers; each
// thread forms the block's 4 x 4 dots and adds them times the block's scales, as the
// reference does per block.
//
// Split-K without a workspace: when the tiles alone would leave SMs idle, a cluster of ks
// CTAs (1 x 1 x ks) takes one tile, each CTA a contiguous range of k blocks; the CTAs then
// leave their partial tiles in shared memory and each reduces its share of the rows over the
// cluster's CTAs in rank order through distributed shared memory (deterministic), and writes
// the epilogue. The kernel has no spin waits: only block and cluster barriers, which every
// thread reaches.
//
// The SiLU pair (the gate and up projections and ops.siluMul of an LLM layer, src/llm.zig:
// 206-208, src/ops.zig:435-440) runs on the same tiles: a tile's 64 columns are 32 gate rows
// and the same 32 up rows, a thread owns two of each, and the epilogue writes
// gate / (1 + exp(-gate)) * up.
//
// Launched as a programmatic dependent (chain.cuh): the weight rows of the CTA's k range are
// prefetched into L2 before the wait for the kernel that wrote x.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "chain.cuh"
#include "common.cuh"
#include "kernels.h"

namespace zwg {

namespace q8g {

constexpr int BM = 32, BN = 64, BK = 32, THREADS = 128, MAX_KS = 8;

struct Smem {
    float xs[2][BK][BM];  // x block, k-major
    float wq[2][BK][BN];  // int8 weights of the block as floats, k-major
    float sc[2][BN];      // the block's scale of each column
    float red[BM][BN];    // this CTA's partial tile (split-K)
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

// The second matrix of the SiLU pair, and its bias.
struct Second {
    const int8_t* wq;
    const float* ws;
    const float* bias;
};

// Column of the tile held by output j (0..3) of thread tx: four consecutive columns, or for
// the SiLU pair two gate columns and the same two up columns.
template <bool PAIR>
__device__ __forceinline__ int tile_col(int tx, int j) {
    return PAIR ? (j < 2 ? tx * 2 + j : BN / 2 + tx * 2 + (j - 2)) : tx * 4 + j;
}

// MODE: LIN_STORE / LIN_ADD / LIN_GELU; PAIR: the SiLU pair (out [m][n], n = n_ff).
template <int MODE, bool PAIR>
__global__ void __launch_bounds__(THREADS) q8_gemm_kernel(const float* x, int m, int k, const int8_t* __restrict__ wq,
                                                          const float* __restrict__ ws, const float* __restrict__ bias,
                                                          int n, float* out, int ks, Second sec) {
    __shared__ __align__(16) Smem sm;
    const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
    // a tile's first output column: 64 columns, or 32 gate / up pairs
    const int n0 = blockIdx.x * (PAIR ? BN / 2 : BN), m0 = blockIdx.y * BM, kz = blockIdx.z;
    const int nb = k / BK;
    const int b_beg = (int)((long long)kz * nb / ks), b_end = (int)((long long)(kz + 1) * nb / ks);
    // loader roles: x rows (t >> 3) and (t >> 3) + 16, four k at (t & 7) * 4; weight row t >> 1,
    // sixteen k at (t & 1) * 16
    const int xrow = t >> 3, xk = (t & 7) * 4, wj = t >> 1, wh = t & 1;
    const bool up = PAIR && wj >= BN / 2;          // this loader's row comes from the up matrix
    const int wn = PAIR ? n0 + (up ? wj - BN / 2 : wj) : n0 + wj;
    const bool wrow_ok = wn < n;
    const int8_t* wrow = (up ? sec.wq : wq) + (size_t)(wrow_ok ? wn : 0) * k;
    const float* wsc = (up ? sec.ws : ws) + (size_t)(wrow_ok ? wn : 0) * nb;
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
                    if (col < n) finish_pair(out, bias, sec.bias, n, row, col, acc[i][j], acc[i][2 + j]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int col = n0 + tx * 4 + j;
                    if (col < n) finish<MODE>(out, bias, n, row, col, acc[i][j]);
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
    for (int e = t; e < rows * OUTS; e += THREADS) {
        const int rr = r0 + e / OUTS, cc = e % OUTS;
        const int row = m0 + rr, col = n0 + cc;
        float v = 0.f, u = 0.f;
        for (int q = 0; q < ks; q++) {
            v = __fadd_rn(v, ld_cluster(cluster_addr(&sm.red[rr][cc], (uint32_t)q)));
            if (PAIR) u = __fadd_rn(u, ld_cluster(cluster_addr(&sm.red[rr][BN / 2 + cc], (uint32_t)q)));
        }
        if (row < m && col < n) {
            if (PAIR) finish_pair(out, bias, sec.bias, n, row, col, v, u);
            else finish<MODE>(out, bias, n, row, col, v);
        }
    }
    // no CTA leaves while another may still read its partial tile
    cluster_sync_all();
}

}  // namespace q8g

namespace {

int launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias, size_t n,
           int mode, bool pair, q8g::Second sec, float* out, int sm_count, cudaStream_t st) {
    using namespace q8g;
    if (m == 0 || n == 0) return 0;
    if (k == 0 || k % BK || ((uintptr_t)x & 15) || ((uintptr_t)wq & 15) || (pair && ((uintptr_t)sec.wq & 15)))
        return -1;
    if (m > (1u << 30) || n > (1u << 30) || k > (1u << 30)) return -1;
    const size_t per_tile = pair ? BN / 2 : BN;
    const size_t tiles_n = (n + per_tile - 1) / per_tile, tiles_m = (m + BM - 1) / BM;
    if (tiles_m > 65535 || tiles_n > 0x7fffffff) return -1;
    const size_t nb = k / BK;
    // k splits (powers of two, at most 8, at least two k blocks each) while the tiles alone
    // would give fewer than two CTAs per SM
    int ks = 1;
    while (ks < MAX_KS && tiles_n * tiles_m * ks < 2 * (size_t)std::max(1, sm_count) && nb / (2 * ks) >= 2) ks *= 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)ks);
    cfg.blockDim = dim3(THREADS);
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
    cudaError_t e;
    const int im = (int)m, ik = (int)k, in = (int)n;
    if (pair) e = cudaLaunchKernelEx(&cfg, q8_gemm_kernel<LIN_STORE, true>, x, im, ik, wq, ws, bias, in, out, ks, sec);
    else if (mode == LIN_ADD)
        e = cudaLaunchKernelEx(&cfg, q8_gemm_kernel<LIN_ADD, false>, x, im, ik, wq, ws, bias, in, out, ks, sec);
    else if (mode == LIN_GELU)
        e = cudaLaunchKernelEx(&cfg, q8_gemm_kernel<LIN_GELU, false>, x, im, ik, wq, ws, bias, in, out, ks, sec);
    else e = cudaLaunchKernelEx(&cfg, q8_gemm_kernel<LIN_STORE, false>, x, im, ik, wq, ws, bias, in, out, ks, sec);
    return e == cudaSuccess ? 0 : -1;
}

}  // namespace

// out[m][n] (+)= x[m][k] . W^T (meant for m >= 16), k a multiple of 32; mode as
// q8_linear_launch. Returns -1 on a bad argument or a launch failure.
int q8_gemm_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias, size_t n,
                   int mode, float* out, int sm_count, cudaStream_t st) {
    return launch(x, m, k, wq, ws, bias, n, mode, false, q8g::Second{nullptr, nullptr, nullptr}, out, sm_count, st);
}

// out[m][n_ff] = silu(x . Wg^T + bg) * (x . Wu^T + bu), the SiLU pair of q8_pair_launch.
int q8_gemm_silu_launch(const float* x, size_t m, size_t k, const int8_t* wg, const float* sg, const float* bg,
                        const int8_t* wu, const float* su, const float* bu, size_t n_ff, float* out, int sm_count,
                        cudaStream_t st) {
    return launch(x, m, k, wg, sg, bg, n_ff, LIN_STORE, true, q8g::Second{wu, su, bu}, out, sm_count, st);
}

}  // namespace zwg
