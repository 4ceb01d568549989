// Whisper encoder self-attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces the encoder's call of the reference attention (src/encoder.zig:167 ->
// ops.attention, src/ops.zig:593-605 -> attentionEx, src/ops.zig:562-590): per window
// and head, O = softmax(Q K^T / sqrt(64)) V over n_ctx = 1500 frames, non-causal.
//
// One CTA computes a 128-row query tile of one (window, head):
//   warp 0      TMA producer: Q once, then K and V tiles of 128 keys into a 3-stage ring
//               (128-byte swizzle, no multicast);
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma:
//                 S_j = Q K_j^T  (M=128, N=128, K=64; A and B K-major)  -> TMEM S[j % 2]
//                 O  += P_j V_j  (M=128, N=64,  K=128; P K-major, V MN-major) -> TMEM O
//               in the order S_0, S_1, O_0, S_2, O_1, ... so the next scores are computed
//               while the softmax warps work on the current ones;
//   warps 4-7   softmax, one thread per query row (TMEM lane = row): read the row of S,
//               online max in base 2, P = exp2(S * log2e/8 - m) written as bf16 into a
//               swizzled shared-memory tile (the A operand of the second MMA), row sums in
//               f32, O rescaled in TMEM only when the running max grows by more than 2^8
//               (otherwise the stale max is kept; numerator and denominator share it);
//               finally O / l is written to global memory as f32.
// Keys past n_ctx come from the TMA's zero fill and are masked to -inf before the max;
// query rows past n_ctx are computed on zeros and not stored.
//
// Every mbarrier wait is bounded (sm100::mbar_wait): a wait that runs out records
// kErrTimeout in the context's error word and the kernel skips to its teardown.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace zwg {

using namespace sm100;

namespace enc_tc {

constexpr int BM = 128;        // query rows per CTA
constexpr int BN = 128;        // keys per tile
constexpr int D = 64;          // head dim
constexpr int NS = 3;          // K/V pipeline stages
constexpr int THREADS = 256;
constexpr uint32_t TILE_BYTES = BM * D * 2;  // 16 KB: one [128][64] bf16 tile
constexpr uint32_t P_BYTES = BM * BN * 2;    // 32 KB: [128][128] bf16 = two K-major halves
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_S0 = 0, TMEM_S1 = 128, TMEM_O = 256;

struct Smem {
    // 1024-byte aligned tiles (128-byte swizzle atoms)
    uint8_t q[TILE_BYTES];
    uint8_t k[NS][TILE_BYTES];
    uint8_t v[NS][TILE_BYTES];
    uint8_t p[2][P_BYTES];
    uint64_t q_full;
    uint64_t k_full[NS];
    uint64_t v_full[NS];
    uint64_t kv_empty[NS];
    uint64_t s_full[2];
    uint64_t p_full[2];
    uint64_t o_done;
    uint32_t tmem_base;
};

constexpr size_t SMEM_BYTES = sizeof(Smem) + 1024;  // + alignment slack

__global__ void __launch_bounds__(THREADS, 1)
    enc_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, float* __restrict__ out, int n_ctx, int n_head,
                       int* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q_tile = blockIdx.x;
    const int head = blockIdx.y;
    const int item = blockIdx.z;
    const int q0 = q_tile * BM;
    const int n_tiles = (n_ctx + BN - 1) / BN;

    // after a recorded failure the remaining CTAs do nothing (uniform exit, before any
    // barrier or TMEM allocation)
    __shared__ int abort_flag;
    if (threadIdx.x == 0) abort_flag = err ? *(volatile int*)err : 0;
    __syncthreads();
    if (abort_flag) return;

    if (threadIdx.x == 0) {
        mbar_init(&sm.q_full, 1);
        for (int s = 0; s < NS; s++) {
            mbar_init(&sm.k_full[s], 1);
            mbar_init(&sm.v_full[s], 1);
            mbar_init(&sm.kv_empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&sm.s_full[b], 1);
            mbar_init(&sm.p_full[b], 128);
        }
        mbar_init(&sm.o_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&sm.tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tm_q);
            prefetch_tmap(&tm_k);
            prefetch_tmap(&tm_v);
            const int c0 = head * D;
            mbar_arrive_expect_tx(&sm.q_full, TILE_BYTES);
            tma_load_3d(&tm_q, &sm.q_full, sm.q, c0, q0, item);
            for (int j = 0; j < n_tiles; j++) {
                const int s = j % NS;
                if (j >= NS && !mbar_wait(&sm.kv_empty[s], ((j / NS) - 1) & 1, err)) break;
                mbar_arrive_expect_tx(&sm.k_full[s], TILE_BYTES);
                tma_load_3d(&tm_k, &sm.k_full[s], sm.k[s], c0, j * BN, item);
                mbar_arrive_expect_tx(&sm.v_full[s], TILE_BYTES);
                tma_load_3d(&tm_v, &sm.v_full[s], sm.v[s], c0, j * BN, item);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_f16(BM, BN, true, false, false);
            constexpr uint32_t idesc_o = idesc_f16(BM, D, true, false, true);
            const uint32_t q_addr = smem_u32(sm.q);
            bool ok = mbar_wait(&sm.q_full, 0, err);
            // S_j = Q K_j^T: four K=16 steps along the head dim inside the 128-byte rows
            auto issue_s = [&](int j) -> bool {
                const int s = j % NS;
                if (!mbar_wait(&sm.k_full[s], (j / NS) & 1, err)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sm.k[s]);
                const uint32_t d_tmem = tmem + ((j & 1) ? TMEM_S1 : TMEM_S0);
#pragma unroll
                for (int kk = 0; kk < D / 16; kk++) {
                    const uint64_t a = smem_desc_sw128(q_addr + kk * 32, 16, 1024);
                    const uint64_t b = smem_desc_sw128(k_addr + kk * 32, 16, 1024);
                    mma_f16_ss(d_tmem, a, b, idesc_s, kk > 0);
                }
                mma_commit(&sm.s_full[j & 1]);
                return true;
            };
            // O += P_j V_j: eight K=16 steps along the keys; P in two 64-key halves
            auto issue_o = [&](int j) -> bool {
                const int s = j % NS;
                if (!mbar_wait(&sm.p_full[j & 1], (j >> 1) & 1, err)) return false;
                if (!mbar_wait(&sm.v_full[s], (j / NS) & 1, err)) return false;
                tc_fence_after();
                const uint32_t p_addr = smem_u32(sm.p[j & 1]);
                const uint32_t v_addr = smem_u32(sm.v[s]);
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++) {
                    const uint64_t a = smem_desc_sw128(p_addr + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
                    const uint64_t b = smem_desc_sw128(v_addr + kk * 16 * 128, 8192, 1024);
                    mma_f16_ss(tmem + TMEM_O, a, b, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&sm.kv_empty[s]);
                mma_commit(&sm.o_done);
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 1; ok && j <= n_tiles; j++) {
                if (j < n_tiles) ok = issue_s(j);
                if (ok) ok = issue_o(j - 1);
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax warps
        const int row = (warp - 4) * 32 + lane;                 // TMEM lane = query row
        const uint32_t lane_addr = (uint32_t)((warp - 4) * 32) << 16;
        const float c = 1.4426950408889634f * 0.125f;           // log2(e) / sqrt(64)
        float m = -INFINITY;                                    // running max, base-2 units
        float l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_tiles && ok; j++) {
            const int b = j & 1;
            if (!mbar_wait(&sm.s_full[b], (j >> 1) & 1, err)) { ok = false; break; }
            tc_fence_after();
            uint32_t sr[BN];
#pragma unroll
            for (int cc = 0; cc < BN / 32; cc++) {
                uint32_t tmp[32];
                tmem_ld32(tmem + lane_addr + (b ? TMEM_S1 : TMEM_S0) + cc * 32, tmp);
#pragma unroll
                for (int i = 0; i < 32; i++) sr[cc * 32 + i] = tmp[i];
            }
            tmem_ld_wait();
            const int valid = n_ctx - j * BN;                   // keys present in this tile
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < BN; i++) {
                float x = __uint_as_float(sr[i]);
                if (i >= valid) x = -INFINITY;
                sr[i] = __float_as_uint(x);
                mx = fmaxf(mx, x);
            }
            const float m_tile = mx * c;
            // P buffer b and the O accumulator are free once O_{j-1} has completed
            if (j > 0) {
                if (!mbar_wait(&sm.o_done, (j - 1) & 1, err)) { ok = false; break; }
                tc_fence_after();
            }
            if (j == 0) {
                m = m_tile;
            } else if (m_tile > m + 8.0f) {
                const float corr = exp2_approx(m - m_tile);
                l *= corr;
#pragma unroll
                for (int cc = 0; cc < D / 32; cc++) {
                    uint32_t o[32];
                    tmem_ld32(tmem + lane_addr + TMEM_O + cc * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
                    tmem_st32(tmem + lane_addr + TMEM_O + cc * 32, o);
                }
                tmem_st_wait();
                m = m_tile;
            }
            // probabilities -> bf16, 128-byte swizzled K-major rows: 16-byte chunk c of
            // row r in 64-key half h lands at chunk (c ^ (r & 7)) of that row
            uint8_t* pbase = sm.p[b];
            const float neg_m = -m;
#pragma unroll
            for (int ch = 0; ch < BN / 8; ch++) {
                uint32_t packed[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float p0 = exp2_approx(fmaf(__uint_as_float(sr[ch * 8 + 2 * e]), c, neg_m));
                    const float p1 = exp2_approx(fmaf(__uint_as_float(sr[ch * 8 + 2 * e + 1]), c, neg_m));
                    l += p0 + p1;
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
                    packed[e] = *reinterpret_cast<uint32_t*>(&h2);
                }
                const int half = ch >> 3, cir = ch & 7;
                uint8_t* dst = pbase + half * (BM * 128) + row * 128 + ((cir ^ (row & 7)) << 4);
                *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&sm.p_full[b]);
        }
        // ---- epilogue: O / l -> out[item][q0 + row][head * 64 ..]
        if (ok && mbar_wait(&sm.o_done, (n_tiles - 1) & 1, err)) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            const int grow = q0 + row;
            float* orow = out + ((size_t)item * n_ctx + grow) * (size_t)(n_head * D) + head * D;
#pragma unroll
            for (int cc = 0; cc < D / 32; cc++) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_addr + TMEM_O + cc * 32, o);
                tmem_ld_wait();
                if (grow < n_ctx) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float4 v4 = make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                                                __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
                        *reinterpret_cast<float4*>(orow + cc * 32 + i) = v4;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace enc_tc

// ---- host side -----------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// 3-d map over a bf16 [n_batch][n_ctx][n_head*64] tensor with [1][128][64] boxes.
static bool make_map(CUtensorMap* map, const void* base, int n_batch, int n_ctx, int n_head) {
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return false;
    const cuuint64_t row = (cuuint64_t)n_head * 64;
    cuuint64_t dims[3] = {row, (cuuint64_t)n_ctx, (cuuint64_t)n_batch};
    cuuint64_t strides[2] = {row * 2, row * 2 * (cuuint64_t)n_ctx};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int enc_tc_launch(const EncTcParams& p, cudaStream_t st) {
    using namespace enc_tc;
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, p.q, p.n_batch, p.n_ctx, p.n_head) || !make_map(&mk, p.k, p.n_batch, p.n_ctx, p.n_head) ||
        !make_map(&mv, p.v, p.n_batch, p.n_ctx, p.n_head))
        return -1;
    // the shared-memory opt-in is a per-device function attribute
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[dev]) {
            if (cudaFuncSetAttribute(enc_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)SMEM_BYTES) != cudaSuccess)
                return -1;
            attr_set[dev] = true;
        }
    }
    dim3 grid((unsigned)((p.n_ctx + BM - 1) / BM), (unsigned)p.n_head, (unsigned)p.n_batch);
    enc_attn_tc_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(mq, mk, mv, p.out, p.n_ctx, p.n_head, p.err);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace zwg
