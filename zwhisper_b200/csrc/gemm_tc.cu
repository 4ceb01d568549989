// The Whisper encoder's dense products as f16 GEMMs on the 5th-generation tensor cores
// (sm_100a): the conv front-end (src/encoder.zig:125-150, each kernel-3 convolution as one
// product over three consecutive input rows), the q/k/v and output projections and the MLP
// (src/encoder.zig:152-176; ops.linear, src/ops.zig:243-306).
//
//   D[b][m][n] = epilogue( sum_k A[b][m][k] * W[n][k] )
//
// A: f16 activations [batch][M][K] (row m of batch b at A + b * a_bs + m * lda); W: f16
// weights [N][K] row-major, the layout of the model file's linear weights; both K-major,
// read by TMA in [rows][64] boxes with the 128-byte swizzle. The reference widens its f16
// weights to f32 and multiplies in f32; here the weights enter the tensor cores exactly and
// the activations are rounded to f16 (11 significant bits), with f32 accumulation.
//
// Persistent kernel over CTA pairs (clusters of 2, tcgen05 cta_group::2), one CTA per SM:
// a pair computes a 256 x 256 tile, each CTA holding 128 rows of A and 128 rows of W in its
// shared memory (32 KB a stage, 6 stages), so a CTA pulls half the W bytes a single-CTA
// 128 x 256 tile would for the same products. Tiles are dealt round-robin over the pairs (n
// fastest, so pairs running together share their A rows through L2).
//   warp 0     TMA producer in both CTAs: its A and W boxes of each 64-wide k step, counted
//              on the first CTA's full barrier (cta_group::2 loads, no multicast).
//   warp 1     allocates 512 TMEM columns in both CTAs (two accumulators of 256); lane 0 of
//              the first CTA issues tcgen05.mma.cta_group::2 kind::f16 (M 256, N 256, K 16)
//              into the accumulator of the tile, alternating between the two, so the
//              epilogue of one tile overlaps the products of the next; its commits arrive
//              in both CTAs.
//   warps 2-9  epilogue in both CTAs, one thread per row of the CTA's 128 (TMEM lane = row)
//              and half of the columns: 32 columns at a time from TMEM, + bias, optional
//              tanh GELU, optional addend (the positional embedding) or accumulation into
//              the f32 output (the residual stream), loaded a chunk ahead; stored as f32, f16
//              or bf16. Rows past M (per batch) and columns past N are not stored. Each warp
//              then releases the accumulator on the first CTA's barrier.
// Every mbarrier wait is bounded; on a timeout the error word is set and the CTA goes to
// the teardown: both CTAs meet at a cluster barrier (every path reaches it) after the first
// CTA has drained its products and copies, then free their TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace zwg {

using namespace sm100;

namespace gemm_tc {

constexpr int BM = 128;        // rows per CTA (M = 256 per pair)
constexpr int BN = 256;        // columns per pair tile (each CTA loads 128 rows of W)
constexpr int BK = 64;         // 64 f16 = one 128-byte swizzled row
constexpr int NS = 5;          // pipeline stages
constexpr int THREADS = 320;   // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;
constexpr uint32_t STAGE_TX = 2 * (A_BYTES + B_BYTES);  // both CTAs' loads, on the first CTA's barrier
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr int EPI_WARPS = 8;

struct Smem {
    uint8_t a[NS][A_BYTES];  // 1024-byte aligned stages
    uint8_t b[NS][B_BYTES];
    float stage[EPI_WARPS][32][33];  // per epilogue warp: a 32 x 32 chunk, rows to columns
    uint64_t full[NS], empty[NS];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort_flag;
};
constexpr size_t SMEM_BYTES = sizeof(Smem) + 1024;

struct Geo {
    int M, N, K, n_batch;
    int m_pairs, n_tiles, k_steps;
    long long total;
};

// Tile t of the pair grid: batch b, first row of the pair's 256, first column.
__device__ __forceinline__ void tile_of(long long t, const Geo& g, int& b, int& m0, int& n0) {
    const long long mt = t / g.n_tiles;
    n0 = (int)(t - mt * g.n_tiles) * BN;
    b = (int)(mt / g.m_pairs);
    m0 = (int)(mt - (long long)b * g.m_pairs) * (2 * BM);
}

// ggml's tanh GELU (src/ops.zig:312-327), 0.5 x (1 + tanh(u)) with u = sqrt(2/pi) (x + 0.044715
// x^3), evaluated through the identity 1 + tanh(u) = 2 / (1 + exp(-2u)) as x / (1 + 2^t) with
// t = -2 log2(e) u = x (K1 + K2 x^2): one base-2 exponential and one reciprocal on the MUFU,
// three other operations. The error is a few ulp of f32 relative to the result (for
// negative x too, where the result is small), far below the f16 or bf16 rounding of the next
// product's operand. Large |x| gives x or -0 exactly.
__device__ __forceinline__ float gelu_fast(float x) {
    constexpr float K1 = -2.0 * 1.4426950408889634 * 0.7978845608028654;  // -2 log2(e) sqrt(2/pi)
    constexpr float K2 = K1 * 0.044715;
    const float t = x * fmaf(K2, x * x, K1);
    return __fdividef(x, 1.0f + exp2_approx(t));
}

// SRC: what is added after the activation: SRC_NONE, SRC_ACC (the f32 output itself, the
// residual stream) or SRC_ADDEND (e.addend, the positional embedding).
enum { SRC_NONE = 0, SRC_ACC = 1, SRC_ADDEND = 2 };

template <int OUT, bool GELU, int SRC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w, Geo geo,
                    GemmEpilogue e, int* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();      // 0: the pair's first CTA (issues the MMAs)
    const long long pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&sm.acc_full[b], 1);
            mbar_init(&sm.acc_empty[b], 2 * EPI_WARPS);
        }
        mbar_init(&sm.mma_done, 1);
        fence_mbar_init();
        sm.abort_flag = err ? *(volatile int*)err : 0;
    }
    if (warp == 1) {
        tmem_alloc_pair(&sm.tmem_base, TMEM_COLS);
        tmem_relinquish_pair();
    }
    // both CTAs' barriers are initialised and their TMEM allocated before any cross-CTA use
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const bool run = sm.abort_flag == 0;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producers
        if (lane == 0 && run) {
            prefetch_tmap(&tm_a);
            prefetch_tmap(&tm_w);
            uint32_t g = 0;
            bool ok = true;
            for (long long t = pair; ok && t < geo.total; t += n_pairs) {
                int b, m0, n0;
                tile_of(t, geo, b, m0, n0);
                for (int ks = 0; ks < geo.k_steps; ks++, g++) {
                    const uint32_t s = g % NS;
                    if (g >= NS && !(ok = mbar_wait(&sm.empty[s], ((g / NS) - 1) & 1, err))) break;
                    const uint32_t fb = mapa_shared(smem_u32(&sm.full[s]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], STAGE_TX);
                    tma_load_3d_pair(&tm_a, fb, sm.a[s], ks * BK, m0 + (int)rank * BM, b);
                    tma_load_3d_pair(&tm_w, fb, sm.b[s], ks * BK, n0 + (int)rank * (BN / 2), 0);
                }
            }
            // every load of both CTAs lands on the first CTA's full barriers: it waits for the
            // last phase of each stage before the teardown
            if (rank == 0)
                for (uint32_t s = 0; s < NS && s < g; s++) mbar_wait_drain(&sm.full[s], ((g - 1 - s) / NS) & 1);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && rank == 0 && run) {
            constexpr uint32_t idesc = idesc_f16(2 * BM, BN, false, false, false);
            uint32_t g = 0;
            int it = 0;
            bool ok = true;
            for (long long t = pair; ok && t < geo.total; t += n_pairs, it++) {
                const int buf = it & 1;
                if (it >= 2 && !(ok = mbar_wait(&sm.acc_empty[buf], ((it >> 1) - 1) & 1, err))) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * BN;
                for (int ks = 0; ks < geo.k_steps; ks++, g++) {
                    const uint32_t s = g % NS;
                    if (!(ok = mbar_wait(&sm.full[s], (g / NS) & 1, err))) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sm.a[s]), b_addr = smem_u32(sm.b[s]);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint64_t ad = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(b_addr + kk * 32, 16, 1024);
                        mma_f16_ss_pair(d, ad, bd, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit_pair(&sm.empty[s]);
                }
                if (ok) mma_commit_pair(&sm.acc_full[buf]);
            }
            // every product has completed (and read both CTAs' shared memory) before the
            // teardown
            mma_commit_pair(&sm.mma_done);
            mbar_wait_drain(&sm.mma_done, 0);
        }
    } else if (run) {
        // ---------------------------------------------------------------- epilogue
        // warps 2-9: two warps per TMEM lane quarter, each taking one half of the columns
        const int quarter = warp & 3;               // TMEM lanes this warp may access
        const int half = (warp - 2) >> 2;           // column half of the tile
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        constexpr int CH = BN / 64;                 // 32-column chunks per half
        // a chunk leaves TMEM one row per lane and goes out through shared memory as four
        // rows per instruction, eight lanes per row, so global reads and writes are whole
        // 128-byte lines
        float (*stg)[33] = sm.stage[warp - 2];
        const int rsub = lane >> 3, q = 4 * (lane & 7);
        constexpr bool has_src = SRC != SRC_NONE;
        int it = 0;
        for (long long t = pair; t < geo.total; t += n_pairs, it++) {
            const int buf = it & 1;
            int b, m0, n0;
            tile_of(t, geo, b, m0, n0);
            const int mw = m0 + (int)rank * BM + quarter * 32;  // first row of this warp's 32
            const int nb = n0 + half * (BN / 2);
            // the f32 values added after the activation (the residual stream or the addend)
            // are loaded one chunk ahead, the first before the accumulator is ready
            auto src_row = [&](int m) -> const float* {
                return SRC == SRC_ACC ? static_cast<const float*>(e.out) + (size_t)b * e.out_bs + (size_t)m * e.ld_out
                                      : e.addend + (size_t)m * e.ld_add;
            };
            float4 cur[8], nxt[8];
            if (has_src && nb < geo.N) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int m = mw + i * 4 + rsub;
                    if (m < geo.M) cur[i] = *reinterpret_cast<const float4*>(src_row(m) + nb + q);
                }
            }
            if (!mbar_wait_warp(&sm.acc_full[buf], (it >> 1) & 1, err)) break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < CH; c++) {
                const int n = nb + c * 32;
                if (n >= geo.N) break;  // uniform over the warp
                if (has_src && c + 1 < CH && n + 32 < geo.N) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int m = mw + i * 4 + rsub;
                        if (m < geo.M) nxt[i] = *reinterpret_cast<const float4*>(src_row(m) + n + 32 + q);
                    }
                }
                uint32_t r[32];
                tmem_ld32(tmem + lane_addr + buf * BN + half * (BN / 2) + c * 32, r);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (e.bias) bb = __ldg(reinterpret_cast<const float4*>(e.bias + n + i));
                    float v0 = __fadd_rn(__uint_as_float(r[i]), bb.x);
                    float v1 = __fadd_rn(__uint_as_float(r[i + 1]), bb.y);
                    float v2 = __fadd_rn(__uint_as_float(r[i + 2]), bb.z);
                    float v3 = __fadd_rn(__uint_as_float(r[i + 3]), bb.w);
                    if (GELU) {
                        v0 = gelu_fast(v0);
                        v1 = gelu_fast(v1);
                        v2 = gelu_fast(v2);
                        v3 = gelu_fast(v3);
                    }
                    stg[lane][i] = v0;
                    stg[lane][i + 1] = v1;
                    stg[lane][i + 2] = v2;
                    stg[lane][i + 3] = v3;
                }
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int rr = i * 4 + rsub;
                    const int m = mw + rr;
                    if (m < geo.M) {
                        float4 x = make_float4(stg[rr][q], stg[rr][q + 1], stg[rr][q + 2], stg[rr][q + 3]);
                        if (has_src)
                            x = make_float4(__fadd_rn(x.x, cur[i].x), __fadd_rn(x.y, cur[i].y), __fadd_rn(x.z, cur[i].z),
                                            __fadd_rn(x.w, cur[i].w));
                        const size_t o = (size_t)b * e.out_bs + (size_t)m * e.ld_out + n + q;
                        if (OUT == GEMM_OUT_F32) {
                            *reinterpret_cast<float4*>(static_cast<float*>(e.out) + o) = x;
                        } else if (OUT == GEMM_OUT_F16) {
                            __half2 h0 = __floats2half2_rn(x.x, x.y), h1 = __floats2half2_rn(x.z, x.w);
                            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(e.out) + o) =
                                make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
                        } else {
                            __nv_bfloat162 h0 = __floats2bfloat162_rn(x.x, x.y), h1 = __floats2bfloat162_rn(x.z, x.w);
                            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(e.out) + o) =
                                make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
                        }
                    }
                }
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 8; i++) cur[i] = nxt[i];
            }
            // the accumulator is in registers or stored: the next tile may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&sm.acc_empty[buf]), 0));
        }
    }

    // teardown: the first CTA's products and copies are drained; neither CTA leaves while the
    // other may still touch its shared memory or TMEM
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, TMEM_COLS);
    }
}

// 3-d map over f16 [dim2][dim1][dim0] with row stride ld and plane stride ps (elements) and
// [1][rows][64] boxes in the 128-byte swizzle; reads outside the extents fill zeros.
static bool make_map(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t dim2, uint64_t ld,
                     uint64_t ps, uint32_t rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {dim0, dim1, dim2};
    cuuint64_t strides[2] = {ld * 2, ps * 2};
    cuuint32_t box[3] = {64, rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gemm_tc

bool gemm_f16_supported(const GemmParams& p) {
    const uintptr_t base = (uintptr_t)p.a | (uintptr_t)p.w;
    if (base & 15) return false;
    if (!p.e.out || ((uintptr_t)p.e.out & 15)) return false;
    if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.n_batch <= 0) return false;
    if (p.N % 32 || p.K % 8 || p.lda % 8 || p.a_bs % 8 || p.ldw % 8) return false;
    if (p.ldw < (size_t)p.K) return false;  // rows of a may overlap (the convolutions' views)
    // 16-byte aligned output rows and chunks; f32 accumulation only into f32 outputs
    const size_t esz = p.out_type == GEMM_OUT_F32 ? 4 : 2;
    if ((p.e.ld_out * esz) % 16 || (p.e.out_bs * esz) % 16) return false;
    if (p.accumulate && (p.out_type != GEMM_OUT_F32 || p.e.addend)) return false;
    if (p.e.addend && p.out_type != GEMM_OUT_F32) return false;
    if (p.e.bias && ((uintptr_t)p.e.bias & 15)) return false;
    if (p.e.addend && (((uintptr_t)p.e.addend & 15) || p.e.ld_add % 4)) return false;
    if (p.out_type < GEMM_OUT_F32 || p.out_type > GEMM_OUT_BF16) return false;
    return true;
}

int gemm_f16_launch(const GemmParams& p, int sm_count, int* err, cudaStream_t st) {
    using namespace gemm_tc;
    if (!gemm_f16_supported(p)) return -1;
    CUtensorMap ma, mw;
    if (!make_map(&ma, p.a, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)p.n_batch, p.lda, p.a_bs ? p.a_bs : p.lda * p.M,
                  BM) ||
        !make_map(&mw, p.w, (uint64_t)p.K, (uint64_t)p.N, 1, p.ldw, p.ldw * (uint64_t)p.N, BN / 2))
        return -1;
    Geo g;
    g.M = p.M;
    g.N = p.N;
    g.K = p.K;
    g.n_batch = p.n_batch;
    g.m_pairs = (p.M + 2 * BM - 1) / (2 * BM);
    g.n_tiles = (p.N + BN - 1) / BN;
    g.k_steps = (p.K + BK - 1) / BK;
    g.total = (long long)g.m_pairs * g.n_batch * g.n_tiles;
    auto go = [&](auto kern) -> int {
        // once per device and kernel: the shared-memory opt-in and the number of CTA pairs
        // that can be resident at once (the SMs of a cluster must share a GPC)
        static std::mutex mu;
        static std::map<std::pair<int, const void*>, int> pairs_of;
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return -1;
        int max_pairs = 0;
        {
            std::lock_guard<std::mutex> lk(mu);
            const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kern));
            const auto it = pairs_of.find(key);
            if (it != pairs_of.end()) {
                max_pairs = it->second;
            } else {
                if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) !=
                    cudaSuccess)
                    return -1;
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3(2 * (unsigned)std::max(1, sm_count / 2));
                cfg.blockDim = dim3(THREADS);
                cfg.dynamicSmemBytes = SMEM_BYTES;
                if (cudaOccupancyMaxActiveClusters(&max_pairs, kern, &cfg) != cudaSuccess || max_pairs < 1)
                    max_pairs = std::max(1, sm_count / 2);
                cudaGetLastError();
                pairs_of[key] = max_pairs;
            }
        }
        const int grid = 2 * (int)std::min<long long>(g.total, max_pairs);
        kern<<<grid, THREADS, SMEM_BYTES, st>>>(ma, mw, g, p.e, err);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    };
    if (p.out_type == GEMM_OUT_F32) {
        if (p.accumulate)
            return p.gelu ? go(gemm_f16_kernel<GEMM_OUT_F32, true, SRC_ACC>) : go(gemm_f16_kernel<GEMM_OUT_F32, false, SRC_ACC>);
        if (p.e.addend)
            return p.gelu ? go(gemm_f16_kernel<GEMM_OUT_F32, true, SRC_ADDEND>)
                          : go(gemm_f16_kernel<GEMM_OUT_F32, false, SRC_ADDEND>);
        return p.gelu ? go(gemm_f16_kernel<GEMM_OUT_F32, true, SRC_NONE>) : go(gemm_f16_kernel<GEMM_OUT_F32, false, SRC_NONE>);
    }
    // 16-bit outputs take no addend (gemm_f16_supported)
    if (p.out_type == GEMM_OUT_F16)
        return p.gelu ? go(gemm_f16_kernel<GEMM_OUT_F16, true, SRC_NONE>) : go(gemm_f16_kernel<GEMM_OUT_F16, false, SRC_NONE>);
    return p.gelu ? go(gemm_f16_kernel<GEMM_OUT_BF16, true, SRC_NONE>) : go(gemm_f16_kernel<GEMM_OUT_BF16, false, SRC_NONE>);
}

}  // namespace zwg
