// Whisper encoder self-attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces the encoder's call of the reference attention (src/encoder.zig:167 ->
// ops.attention, src/ops.zig:593-605 -> attentionEx, src/ops.zig:562-590): per window
// and head, O = softmax(Q K^T / sqrt(64)) V over n_ctx = 1500 frames, non-causal.
//
// Persistent kernel, one CTA per SM. A work item is a pair of 128-row query tiles of one
// (window, head); items are dealt round-robin to the CTAs, pairs of one head first so CTAs
// running together read the same K/V through L2.
//   warp 0      TMA producer: both Q tiles of an item (double-buffered across items), then
//               K and V tiles of 128 keys into a 3-stage ring (128-byte swizzle, no
//               multicast).
//   warps 1-2   warp 1 allocates 512 TMEM columns; lane 0 of warp 1 + t issues the
//               tcgen05.mma (kind::f16, bf16) of query tile t:
//                 S_t = Q_t K_j^T  (M=128, N=128, K=64; A, B K-major from shared memory)
//                 O_t += P_t V_j   (M=128, N=64, K=128; P from TMEM, V MN-major in smem)
//               for the two query tiles t = 0, 1. The next scores S_t(j+1) are issued as soon
//               as the softmax has copied S_t(j) into registers (P has its own columns), so
//               the tensor core computes them while the exponentials of tile j run; the PV
//               of tile j follows when P_t(j) is written.
//   warp 3      idle (it completes the control warpgroup for the register split);
//   warps 4-11  two softmax warpgroups, one per query tile, one thread per query row (TMEM
//               lane = row): read the 128 scores of the row (then release the score columns
//               to the next S), online max in base 2, P = exp2(S * c - m) packed to bf16 and
//               stored into the tile's P columns (the A operand of the PV MMA) once the
//               previous PV has read them, f32 row sums, O rescaled in TMEM only when the
//               running max grows by more than 2^8 (otherwise the stale max is kept:
//               numerator and denominator share it); after the last tile, O / l goes out
//               by TMA stores staged in the item's Q tile buffer (the epilogue below).
// TMEM columns per query tile t: S at 256t (128), P at 256t + 128 (64 columns of bf16
// pairs), O at 256t + 192 (64); the two tiles fill all 512.
// Keys past n_ctx come from the TMA's zero fill and are masked to -inf before the max; query
// rows past n_ctx are computed on zeros and not stored.
//
// Every mbarrier wait is bounded (sm100::mbar_wait): a wait that runs out records
// kErrTimeout in the context's error word, the CTA skips to its teardown, and CTAs that
// start later see the error word and exit at once.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace zwg {

using namespace sm100;

namespace enc_tc {

constexpr int BM = 128;        // query rows per tile
constexpr int BN = 128;        // keys per tile
static_assert(BN == 128, "a softmax row is one 128-column TMEM load and one 64-column store");
constexpr int D = 64;          // head dim
constexpr int NS = 3;          // K/V pipeline stages
constexpr int THREADS = 384;   // 12 warps: control warpgroup + two softmax warpgroups
// Register split (setmaxnreg): launched at 168 per thread (65536 / 384, rounded down to a
// multiple of 8) = 64512 in all; the control warpgroup gives back to 56 and the two softmax
// warpgroups take 224: 128 * 56 + 256 * 224 = 64512, the launch total exactly.
constexpr uint32_t REGS_CONTROL = 56;
constexpr uint32_t REGS_SOFTMAX = 224;
static_assert(128 * REGS_CONTROL + 256 * REGS_SOFTMAX <= THREADS * 168, "register split exceeds the launch");
constexpr uint32_t TILE_BYTES = BM * D * 2;  // 16 KB: one [128][64] bf16 tile
constexpr uint32_t TMEM_COLS = 512;
// per query tile t: scores at 256t, probabilities (bf16 pairs) at 256t + 128, O at 256t + 192
__host__ __device__ constexpr uint32_t s_col(int t) { return t ? 256u : 0u; }
__host__ __device__ constexpr uint32_t p_col(int t) { return t ? 384u : 128u; }
__host__ __device__ constexpr uint32_t o_col(int t) { return t ? 448u : 192u; }

// Pairs of exponentials per 16 (per 32 columns) evaluated by exp2_poly2 on the FMA pipe;
// the others use the MUFU ex2. MUFU is the limit of a d=64 attention (16 exponentials per
// clock per SM against 128 FMA lanes), so part of the work moves to the FMA pipe. Measured
// on B200 (small.en, 64 windows): 0 -> 0.660 ms, 2 -> 0.630, 3 and 4 -> 0.621, 5 -> 0.632,
// 6 -> 0.643, 8 -> 0.674; the output error stays at bf16's (1.03e-3 max-abs on N(0,1) data).
#ifndef ZWG_POLY_PAIRS
#define ZWG_POLY_PAIRS 4
#endif
constexpr int POLY_PAIRS = ZWG_POLY_PAIRS;

struct Smem {
    uint8_t q[2][2][TILE_BYTES];  // [buffer][query tile], 1024-byte aligned tiles
    uint8_t k[NS][TILE_BYTES];
    uint8_t v[NS][TILE_BYTES];
    uint64_t q_full[2], q_empty[2];
    uint64_t k_full[NS], v_full[NS], kv_empty[NS];
    uint64_t s_full[2], s_free[2], p_full[2], pv_done[2];
    uint32_t tmem_base;
    int abort_flag;
};

constexpr size_t SMEM_BYTES = sizeof(Smem) + 1024;  // + alignment slack

__device__ __forceinline__ void decode_item(int item, int n_pairs, int n_head, int& win, int& head, int& pair) {
    pair = item % n_pairs;
    head = (item / n_pairs) % n_head;
    win = item / (n_pairs * n_head);
}

// Epilogue of one warp's 32 rows: O / l is staged in the item's Q tile buffer (4 KB per
// warp, 128-byte rows in the 128-byte swizzle the TMA store reads; the tile's S MMAs have
// all completed by now) and written by TMA stores of [32 rows][32 f32] (two, f32 out) or
// [32 rows][64 f16] (one), whole 128-byte lines, instead of one row per thread. Rows past
// n_ctx fall outside the tensor map and are not written. Lane 0 then waits until the
// stores have read the staging and releases the Q buffer to the producer.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <bool OUT_F16>
__device__ __forceinline__ void write_out(const CUtensorMap* tm_o, Smem& sm, const uint32_t (&o)[64], float l,
                                          int it, int t, int quarter, int lane, int win, int head, int pair) {
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    uint8_t* stage = sm.q[it & 1][t] + quarter * 4096;
    const uint32_t row_addr = smem_u32(stage) + lane * 128;
    const int sw = lane & 7;
    const int row0 = pair * 2 * BM + t * BM + quarter * 32;
    if (OUT_F16) {
#pragma unroll
        for (int c = 0; c < 8; c++) {
            uint32_t h[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                __half2 p2 = __floats2half2_rn(__uint_as_float(o[8 * c + 2 * u]) * inv,
                                               __uint_as_float(o[8 * c + 2 * u + 1]) * inv);
                h[u] = *reinterpret_cast<uint32_t*>(&p2);
            }
            st_shared_v4(row_addr + ((c ^ sw) << 4), h[0], h[1], h[2], h[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_3d(tm_o, stage, head * D, row0, win);
            bulk_commit_group();
        }
    } else {
#pragma unroll
        for (int half = 0; half < 2; half++) {
            if (half) {
                if (lane == 0) bulk_wait_read0();
                __syncwarp();
            }
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const int i = half * 32 + 4 * c;
                st_shared_v4(row_addr + ((c ^ sw) << 4), __float_as_uint(__uint_as_float(o[i]) * inv),
                             __float_as_uint(__uint_as_float(o[i + 1]) * inv),
                             __float_as_uint(__uint_as_float(o[i + 2]) * inv),
                             __float_as_uint(__uint_as_float(o[i + 3]) * inv));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_3d(tm_o, stage, head * D + half * 32, row0, win);
                bulk_commit_group();
            }
        }
    }
    if (lane == 0) {
        bulk_wait_read0();
        mbar_arrive(&sm.q_empty[it & 1]);
    }
    __syncwarp();
}

// OUT_F16: the output is f16 (the operand of the output projection) instead of f32.
template <bool OUT_F16>
__global__ void __launch_bounds__(THREADS, 1)
    enc_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o, int n_ctx, int n_head,
                       int n_items, int* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_tiles = (n_ctx + BN - 1) / BN;          // key tiles (= query tiles)
    const int n_pairs = (n_tiles + 1) / 2;

    // after a recorded failure the remaining CTAs do nothing (uniform exit, before any
    // barrier or TMEM allocation)
    if (threadIdx.x == 0) sm.abort_flag = err ? *(volatile int*)err : 0;
    __syncthreads();
    if (sm.abort_flag) return;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; b++) {
            mbar_init(&sm.q_full[b], 1);
            mbar_init(&sm.q_empty[b], 8);  // lane 0 of every softmax warp, after its output store
            mbar_init(&sm.s_full[b], 1);
            mbar_init(&sm.s_free[b], 128);
            mbar_init(&sm.p_full[b], 128);
            mbar_init(&sm.pv_done[b], 1);
        }
        for (int s = 0; s < NS; s++) {
            mbar_init(&sm.k_full[s], 1);
            mbar_init(&sm.v_full[s], 1);
            mbar_init(&sm.kv_empty[s], 2);  // one commit from each MMA issuer
        }
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

    if (warp < 4) {
      regs_dec<REGS_CONTROL>();
      if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tm_q);
            prefetch_tmap(&tm_k);
            prefetch_tmap(&tm_v);
            uint32_t g = 0;
            int it = 0;
            bool ok = true;
            for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, it++) {
                int win, head, pair;
                decode_item(item, n_pairs, n_head, win, head, pair);
                const int c0 = head * D;
                const int qb = it & 1;
                if (it >= 2 && !(ok = mbar_wait(&sm.q_empty[qb], ((it >> 1) - 1) & 1, err))) break;
                mbar_arrive_expect_tx(&sm.q_full[qb], 2 * TILE_BYTES);
                tma_load_3d(&tm_q, &sm.q_full[qb], sm.q[qb][0], c0, pair * 2 * BM, win);
                tma_load_3d(&tm_q, &sm.q_full[qb], sm.q[qb][1], c0, pair * 2 * BM + BM, win);
                for (int j = 0; j < n_tiles; j++, g++) {
                    const int s = g % NS;
                    if (g >= NS && !(ok = mbar_wait(&sm.kv_empty[s], ((g / NS) - 1) & 1, err))) break;
                    mbar_arrive_expect_tx(&sm.k_full[s], TILE_BYTES);
                    tma_load_3d(&tm_k, &sm.k_full[s], sm.k[s], c0, j * BN, win);
                    mbar_arrive_expect_tx(&sm.v_full[s], TILE_BYTES);
                    tma_load_3d(&tm_v, &sm.v_full[s], sm.v[s], c0, j * BN, win);
                }
            }
        }
      } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------------------ MMA issuers
        // warp 1 issues the MMAs of query tile 0, warp 2 those of tile 1: a thread's MMAs
        // run in issue order, and with one issuer per tile neither tile's instructions
        // wait behind the other tile's barriers.
        if (lane == 0) {
            const int t = warp - 1;
            constexpr uint32_t idesc_s = idesc_f16(BM, BN, true, false, false);
            constexpr uint32_t idesc_o = idesc_f16(BM, D, true, false, true);
            uint32_t g = 0;      // global key-tile counter (phases of the per-tile barriers)
            int it = 0;
            bool ok = true;
            for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, it++) {
                const int qb = it & 1;
                if (!(ok = mbar_wait(&sm.q_full[qb], (it >> 1) & 1, err))) break;
                const uint32_t q_addr = smem_u32(sm.q[qb][t]);
                // S_t(tile gj) = Q_t K^T into the score columns, once the softmax has read the
                // previous scores out of them (s_free of tile gj - 1)
                auto issue_s = [&](uint32_t gj) -> bool {
                    if (!mbar_wait(&sm.k_full[gj % NS], (gj / NS) & 1, err)) return false;
                    if (gj > 0 && !mbar_wait(&sm.s_free[t], (gj - 1) & 1, err)) return false;
                    tc_fence_after();
                    const uint32_t k_addr = smem_u32(sm.k[gj % NS]);
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        const uint64_t a = smem_desc_sw128(q_addr + kk * 32, 16, 1024);
                        const uint64_t b = smem_desc_sw128(k_addr + kk * 32, 16, 1024);
                        mma_f16_ss(tmem + s_col(t), a, b, idesc_s, kk > 0);
                    }
                    mma_commit(&sm.s_full[t]);
                    return true;
                };
                // tile 1 starts one softmax phase behind tile 0, so the two warpgroups'
                // exponential phases alternate on the MUFU instead of coinciding
                if (t == 1 && !(ok = mbar_wait(&sm.p_full[0], g & 1, err))) break;
                ok = issue_s(g);
                for (int j = 0; ok && j < n_tiles; j++) {
                    const uint32_t gj = g + j;
                    const int s = gj % NS;
                    // next scores first: they need only K(j+1) and free score columns
                    if (j + 1 < n_tiles && !(ok = issue_s(gj + 1))) break;
                    // O_t += P_t(j) V(j) once the softmax has written P_t(j)
                    if (!(ok = mbar_wait(&sm.p_full[t], gj & 1, err))) break;
                    if (!(ok = mbar_wait(&sm.v_full[s], (gj / NS) & 1, err))) break;
                    tc_fence_after();
                    const uint32_t v_addr = smem_u32(sm.v[s]);
#pragma unroll
                    for (int kk = 0; kk < BN / 16; kk++) {
                        const uint64_t b = smem_desc_sw128(v_addr + kk * 16 * 128, 8192, 1024);
                        mma_f16_ts(tmem + o_col(t), tmem + p_col(t) + kk * 8, b, idesc_o,
                                   (j > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&sm.pv_done[t]);
                    mma_commit(&sm.kv_empty[s]);
                }
                g += n_tiles;
            }
        }
      }
    } else {
        regs_inc<REGS_SOFTMAX>();
        // ------------------------------------------------------------ softmax warpgroups
        const int t = (warp - 4) >> 2;                  // query tile of this warpgroup
        const int quarter = warp & 3;                   // TMEM lanes this warp may access
        const int row = quarter * 32 + lane;            // TMEM lane = query row in the tile
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        const uint32_t s_addr = tmem + lane_addr + s_col(t);
        const uint32_t p_addr = tmem + lane_addr + p_col(t);
        const uint32_t o_addr = tmem + lane_addr + o_col(t);
        const float c = 1.4426950408889634f * 0.125f;  // log2(e) / sqrt(64)
        uint32_t g = 0;
        int it = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, it++) {
            int win, head, pair;
            decode_item(item, n_pairs, n_head, win, head, pair);
            float m = -INFINITY;                        // running max, base-2 units
            float l = 0.f;
            for (int j = 0; j < n_tiles; j++) {
                const uint32_t gj = g + j;
                if (!(ok = mbar_wait_warp(&sm.s_full[t], gj & 1, err))) break;
                tc_fence_after();
                uint32_t sr[BN];
                tmem_ld128(s_addr, sr);  // the row's 128 scores, one load
                tmem_ld_wait();
                // the scores are in registers: the next S may be written over them
                tc_fence_before();
                mbar_arrive(&sm.s_free[t]);
                const int valid = n_ctx - j * BN;        // keys present in this tile
                if (valid < BN) {
#pragma unroll
                    for (int i = 0; i < BN; i++)
                        if (i >= valid) sr[i] = __float_as_uint(-INFINITY);
                }
                // row max over 8 independent partial maxima, two new scores per three-input max
                float mxp[8];
#pragma unroll
                for (int k = 0; k < 8; k++) mxp[k] = fmaxf(__uint_as_float(sr[k]), __uint_as_float(sr[k + 8]));
#pragma unroll
                for (int i = 16; i < BN; i += 16)
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        mxp[k] = fmax3(mxp[k], __uint_as_float(sr[i + k]), __uint_as_float(sr[i + 8 + k]));
                const float m_tile =
                    fmaxf(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], fmax3(mxp[5], mxp[6], mxp[7]))) * c;
                // the running max is kept stale unless it grows by more than 2^8
                const bool rescale = j > 0 && m_tile > m + 8.0f;
                const float m_old = m;
                if (j == 0 || rescale) m = m_tile;
                const float2 c2 = make_float2(c, c);
                const float2 nm2 = make_float2(-m, -m);
                float2 lp[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                make_float2(0.f, 0.f)};
                uint32_t pk[BN / 2];
#pragma unroll
                for (int e = 0; e < BN / 2; e++) {
                    const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1])),
                                                c2, nm2);
                    // a share of the exponentials can run on the FMA pipe, the rest on MUFU
                    const float2 pr = ((e & 15) < POLY_PAIRS) ? exp2_poly2(x)
                                                             : make_float2(exp2_approx(x.x), exp2_approx(x.y));
                    lp[e & 3] = __fadd2_rn(lp[e & 3], pr);
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(pr.x, pr.y);
                    pk[e] = *reinterpret_cast<uint32_t*>(&h2);
                }
                {
                    const float2 a = __fadd2_rn(lp[0], lp[1]), b = __fadd2_rn(lp[2], lp[3]);
                    const float2 s2 = __fadd2_rn(a, b);
                    const float corr = rescale ? exp2_approx(m_old - m) : 1.f;
                    l = l * corr + (s2.x + s2.y);
                }
                // the previous PV must be done before O is rescaled or P overwritten; the
                // exponentials above ran while it was in flight
                if (j > 0) {
                    if (!(ok = mbar_wait_warp(&sm.pv_done[t], (gj - 1) & 1, err))) break;
                    tc_fence_after();
                }
                // tcgen05.ld/st are warp-collective: the warp rescales if any of its rows
                // must (corr is 1 in the others)
                if (__any_sync(0xffffffffu, rescale)) {
                    const float corr = rescale ? exp2_approx(m_old - m) : 1.f;
#pragma unroll
                    for (int cc = 0; cc < D / 32; cc++) {
                        uint32_t o[32];
                        tmem_ld32(o_addr + cc * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
                        tmem_st32(o_addr + cc * 32, o);
                    }
                }
tmem_st64(p_addr, pk);  // the row's 64 bf16 pairs, one store
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&sm.p_full[t]);
            }
            // ---- epilogue: O / l by TMA stores staged in this item's Q tile buffer
            if (!ok || !(ok = mbar_wait_warp(&sm.pv_done[t], (g + n_tiles - 1) & 1, err))) break;
            tc_fence_after();
            {
                uint32_t o[64];
                tmem_ld64(o_addr, o);
                tmem_ld_wait();
                write_out<OUT_F16>(&tm_o, sm, o, l, it, t, quarter, lane, win, head, pair);
            }
            tc_fence_before();
            g += n_tiles;
        }
    }

    if (warp >= 4 && lane == 0) bulk_wait0();
    // warps whose loops ran in lane 0 alone reach the barrier converged
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace enc_tc

// ---- host side -----------------------------------------------------------------------------

// 3-d map over a bf16 [n_batch][n_ctx][n_head*64] tensor whose rows are ld elements apart,
// with [1][128][64] boxes.
static bool make_map(CUtensorMap* map, const void* base, int n_batch, int n_ctx, int n_head, size_t ld) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    const cuuint64_t row = (cuuint64_t)n_head * 64;
    cuuint64_t dims[3] = {row, (cuuint64_t)n_ctx, (cuuint64_t)n_batch};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)ld * 2 * (cuuint64_t)n_ctx};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static bool make_out_map(CUtensorMap* map, void* base, int n_batch, int n_ctx, int n_head, bool f16) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    const cuuint64_t row = (cuuint64_t)n_head * 64;
    const cuuint64_t esz = f16 ? 2 : 4;
    cuuint64_t dims[3] = {row, (cuuint64_t)n_ctx, (cuuint64_t)n_batch};
    cuuint64_t strides[2] = {row * esz, row * esz * (cuuint64_t)n_ctx};
    cuuint32_t box[3] = {f16 ? 64u : 32u, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int enc_tc_launch(const EncTcParams& p, cudaStream_t st) {
    using namespace enc_tc;
    const size_t ld = p.ld_qkv ? p.ld_qkv : (size_t)p.n_head * 64;
    if (ld < (size_t)p.n_head * 64 || ld % 8) return -1;
    if (((uintptr_t)p.out & 15) != 0) return -1;
    CUtensorMap mq, mk, mv, mo;
    if (!make_map(&mq, p.q, p.n_batch, p.n_ctx, p.n_head, ld) || !make_map(&mk, p.k, p.n_batch, p.n_ctx, p.n_head, ld) ||
        !make_map(&mv, p.v, p.n_batch, p.n_ctx, p.n_head, ld) ||
        !make_out_map(&mo, p.out, p.n_batch, p.n_ctx, p.n_head, p.out_f16 != 0))
        return -1;
    static std::mutex mu;
    static bool attr_set[64][2] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    auto kern = p.out_f16 ? enc_attn_tc_kernel<true> : enc_attn_tc_kernel<false>;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[dev][p.out_f16 ? 1 : 0]) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) != cudaSuccess)
                return -1;
            attr_set[dev][p.out_f16 ? 1 : 0] = true;
        }
    }
    static int sm_count[64] = {};
    if (!sm_count[dev]) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    const int n_tiles = (p.n_ctx + BN - 1) / BN;
    const long long n_items = (long long)p.n_batch * p.n_head * ((n_tiles + 1) / 2);
    if (n_items > (1ll << 30)) return -1;
    const int grid = (int)std::min<long long>(n_items, sm_count[dev] > 0 ? sm_count[dev] : 148);
    kern<<<grid, THREADS, SMEM_BYTES, st>>>(mq, mk, mv, mo, p.n_ctx, p.n_head, (int)n_items, p.err);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace zwg
