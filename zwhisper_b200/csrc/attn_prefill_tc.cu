// Qwen2 prefill attention on tcgen05 tensor cores: causal grouped-query attention of a
// chunk of queries over the transposed f32 key cache, kind::tf32 with f32 accumulation.
//
// Reference: the Qwen2 attention call src/llm.zig:191-202, which runs ops.attentionEx
// (src/ops.zig:517-541, 562-590) with kt_stride = n_ctx over cache_kt[n_head_kv][d][n_ctx]
// and cache_v[n_ctx][n_head_kv*d] (src/llm.zig:27-28, 184-190); query head h reads kv head
// h / (n_head / n_head_kv) (src/ops.zig:521); query i sees keys j <= n_kv - n_q + i. Prefill
// runs the prompt in chunks of up to 256 queries (src/llm.zig:257-266).
//
// Design. The caches stay in the reference's f32 layout; the tensor cores read them as
// tf32 (10-bit mantissa, the low 13 bits of each f32 ignored), so no conversion pass or
// second copy of the cache exists.
//   - A tile is 128 rows = qn consecutive queries x the `group` query heads of one kv head
//     (row = query * group + head-in-group), so one K/V tile feeds every head of the group
//     and the rows of a tile share nearly the same causal limit. Key tiles are 128 wide: a
//     score MMA of N = 128 runs near the full tf32 rate, where N = 64 with an MN-major B
//     operand measured half of it.
//   - Q lives in TMEM (row m in lane m, one f32 per column): the softmax warps load each
//     item's rows from global memory and store them with tcgen05.st, and S = Q K^T is the
//     A-from-TMEM form of tcgen05.mma. Shared memory then holds only the K/V ring.
//   - K^T tiles are [d][128 keys] (four [d][32 keys] boxes): the MN-major B operand of
//     S = Q K^T, read straight from the transposed cache. V tiles are [128 keys][d] (d / 32
//     boxes of [128 keys][32 columns]): the MN-major B operand of O += P V. An MN-major tf32
//     operand must be in the 128-byte swizzle with 32-byte atoms (descriptor layout 1, TMA
//     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B); the 16-byte-atom swizzle that serves K-major
//     operands gives an MMA that writes zeros.
//   - One ring of slots (a K^T or V tile each: three of 64 KB at d = 128, six of 32 KB at
//     d = 64) holds the tiles in the order the MMAs consume them: K0 K1 V0 K2 V1 K3 ...
//     V(n-1). A slot is released by the commit of the MMAs that read it. (Parts of 32 KB
//     released half-way through a tile measured slower at d = 128: 0.46 against 0.34 ms.)
//   - TMEM: Q (d columns), two 128-column score buffers (S of tile j in buffer j % 2; the
//     softmax writes the probabilities P back over the scores as tf32, and P is the TMEM A
//     operand of the PV MMA) and a d-column O accumulator: 512 columns, one CTA per SM.
//   - Warp 0 lane 0: TMA producer. Warp 1: TMEM allocation and the single MMA-issuing
//     thread, order S0 S1 | PV0 S2 | PV1 S3 ...: the next scores are computed while the
//     softmax works on the current ones, and S(j+2) overwrites buffer j % 2 only after PV(j)
//     in issue order (tcgen05.mma from one thread executes in order). Warps 2-5: Q into
//     TMEM, then the softmax, one thread per row (TMEM lane), online max in base 2 kept
//     stale unless it grows by more than 2^8, exp2 on the MUFU, P rounded to tf32 (round to
//     nearest), and the epilogue O / l.
//   - Persistent grid over (sequence, kv head, query tile) items, a pair's tiles adjacent.
//   - d = 64, launches with enough items: two query tiles per item (one score buffer each,
//     a softmax warpgroup each, ring order K0 V0 K1 V1 ..., MMA order S_0(0) S_1(0) | PV_0(j)
//     S_0(j+1) PV_1(j) S_1(j+1) ...), chosen at launch when it needs fewer item-waves by its
//     weight; Cfg below.
// Every wait is bounded; a wait that runs out records kErrTimeout, the CTA drains its own
// copies and MMAs with bounded waits, frees TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace zwg {
namespace prefill_tc {

using namespace sm100;

constexpr int BM = 128;                // rows per tile = TMEM lanes
constexpr int BN = 128;                // keys per tile

// Pairs of exponentials per 16 evaluated by exp2_poly2 on the FMA pipe (relative error
// 1e-4, below tf32's rounding of P); the others use the MUFU ex2, 16 per clock per SM.
// Measured on B200 (last chunk of a 2000-token prompt; ms at d = 128 / d = 64): 0 -> 0.321 /
// 0.0887, 1 -> 0.323 / 0.0882, 2 -> 0.326 / 0.0900, 3 -> 0.335 / 0.0927, 4 -> 0.331 /
// 0.0970, 8 -> 0.344 / 0.1078. With the tf32 rounding done by integer operations the MUFU
// is no longer the limit here (it was: cvt.rna.tf32 shared it with ex2).
constexpr int POLY_PAIRS = 1;

// One CTA per SM with 512 TMEM columns; the ring has three 64 KB slots at d = 128, six
// 32 KB slots at d = 64.
//   d = 128: one query tile per item, two score buffers (S(j+1) is computed while the
//            softmax works on S(j)); warp 0 TMA, warp 1 MMA, warps 2-5 softmax.
//   d = 64:  two query tiles per item (NT = 2) that share every K/V tile, one score buffer
//            each, a softmax warpgroup each (warps 4-7 and 8-11; warps 0-3 are the control
//            warpgroup: 0 TMA, 1 MMA): while one tile's softmax runs, the tensor core works
//            on the other tile, and each K/V tile feeds twice the rows. At d = 64 one query
//            tile's MMAs (S 8 x N128 and PV 16 x N64, the latter at half rate) take ~2,000
//            clocks per key tile against ~1,750 for its softmax, so a single tile per CTA
//            left the tensor core waiting for every P. TMEM per tile: Q 64, S 128, O 64.
template <int D, int NT_ = 1>
struct Cfg {
    static constexpr int NT = NT_;                          // query tiles per item
    static_assert(NT == 1 || D == 64, "two query tiles per item fit TMEM at d = 64 only");
    static constexpr int SBUF = NT == 2 ? 1 : 2;            // score buffers per query tile
    static constexpr int THREADS = NT == 2 ? 384 : 192;
    static constexpr int SM_WARP0 = NT == 2 ? 4 : 2;        // first softmax warp
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t TILE_COLS = TMEM_COLS / NT;   // TMEM columns of one query tile
    static constexpr uint32_t K_CHUNK = D * 128;            // [D rows][32 keys]
    static constexpr uint32_t V_CHUNK = BN * 128;           // [128 keys][32 floats]
    static constexpr uint32_t SLOT = BN * D * 4;            // one K^T or V tile
    static constexpr int NSLOT = D == 128 ? 3 : 6;
    static constexpr uint32_t Q_COL = 0;                    // + tile * TILE_COLS
    static constexpr uint32_t S_COL = D;                    // + tile * TILE_COLS + buffer * BN
    static constexpr uint32_t O_COL = D + SBUF * BN;        // + tile * TILE_COLS
    static_assert(O_COL + D <= TILE_COLS, "TMEM columns");
};

// d = 64 register split (setmaxnreg): launched at 168 per thread (65536 / 384 rounded down
// to a multiple of 8) = 64512; the control warpgroup gives back to 56 and the two softmax
// warpgroups take 224: 128 * 56 + 256 * 224 = 64512, the launch total exactly.
constexpr uint32_t REGS_CONTROL = 56;
constexpr uint32_t REGS_SOFTMAX = 224;
static_assert(128 * REGS_CONTROL + 256 * REGS_SOFTMAX <= Cfg<64, 2>::THREADS * 168, "register split exceeds the launch");

template <int D, int NT_>
struct Smem {
    using C = Cfg<D, NT_>;
    static constexpr int NT = C::NT, SBUF = C::SBUF;
    alignas(1024) uint8_t ring[C::NSLOT][C::SLOT];
    uint64_t full[C::NSLOT], empty[C::NSLOT];
    uint64_t q_full[NT], s_full[NT][SBUF], p_full[NT][SBUF], pv_done[NT][2], drain;
    uint32_t tmem_base;
    int abort_flag;
};

template <int D, int NT>
constexpr size_t smem_bytes() {
    return sizeof(Smem<D, NT>) + 1024;  // + alignment slack
}

struct Args {
    const float* q;
    size_t q_stride, q_bs;
    float* out;
    size_t out_stride, out_bs;
    int n_q, n_kv, n_head_kv, group, qn, rows, n_mt, n_units, n_items, causal;
    int* err;
};

// Consecutive items are the query tiles of one (sequence, kv head), longest causal range
// first: the CTAs running at the same time share that pair's K^T/V tiles through L2, so
// each K/V byte comes from DRAM about once. (Ordering by query tile first made every tile
// re-read its pair's 2 MB of K/V from DRAM: 2.3 GB of DRAM reads for 0.35 GB of inputs in
// a 64-sequence launch.) The static stride over the persistent grid deals each CTA a mix
// of long and short tiles.
// An item is unit u of (sequence b, kv head kh): query tiles u * NT .. u * NT + NT - 1
// (a tile past the last holds no valid rows).
__device__ __forceinline__ void item_of(const Args& a, int idx, int& b, int& kh, int& u) {
    const int bh = idx / a.n_units;
    u = a.n_units - 1 - (idx - bh * a.n_units);
    b = bh / a.n_head_kv;
    kh = bh - b * a.n_head_kv;
}

// Key tiles an item needs: up to the causal limit of the last query of its last tile.
template <int NT>
__device__ __forceinline__ int item_tiles(const Args& a, int u) {
    int keys = a.n_kv;
    if (a.causal) {
        const int last_q = min(min((u + 1) * NT, a.n_mt) * a.qn, a.n_q) - 1;
        keys = min(a.n_kv - a.n_q + last_q + 1, a.n_kv);
    }
    return (keys + BN - 1) / BN;
}

template <int D, int NT>
__global__ void __launch_bounds__(Cfg<D, NT>::THREADS, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const Args a) {
    using C = Cfg<D, NT>;
    constexpr int NS = C::NSLOT;
    extern __shared__ uint8_t smem_raw[];
    Smem<D, NT>& sm = *reinterpret_cast<Smem<D, NT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int* err = a.err;

    // after a recorded failure the remaining CTAs do nothing
    if (threadIdx.x == 0) sm.abort_flag = err ? *(volatile int*)err : 0;
    __syncthreads();
    if (sm.abort_flag) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int t = 0; t < NT; t++) {
            mbar_init(&sm.q_full[t], 128);
            for (int s = 0; s < C::SBUF; s++) {
                mbar_init(&sm.s_full[t][s], 1);
                mbar_init(&sm.p_full[t][s], 128);
            }
            mbar_init(&sm.pv_done[t][0], 1);
            mbar_init(&sm.pv_done[t][1], 1);
        }
        mbar_init(&sm.drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&sm.tmem_base, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp < C::SM_WARP0) {
      if constexpr (NT == 2) regs_dec<REGS_CONTROL>();
      if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        // Loads go into the ring in the order the MMAs first read them (one tile: K0 K1 V0
        // K2 V1 K3 ...; two: K0 V0 K1 V1 ...); at exit (normal or not) the last loads are
        // waited for, so no copy is in flight when the CTA's memory goes.
        if (lane == 0) {
            prefetch_tmap(&tm_k);
            prefetch_tmap(&tm_v);
            uint32_t n = 0;
            bool ok = true;
            auto load = [&](bool is_k, int j, int b, int kh) -> bool {
                const uint32_t slot = n % NS;
                if (n >= (uint32_t)NS && !mbar_wait(&sm.empty[slot], ((n / NS) - 1) & 1, err)) return false;
                mbar_arrive_expect_tx(&sm.full[slot], C::SLOT);
                uint8_t* dst = sm.ring[slot];
                if (is_k) {
#pragma unroll
                    for (int c = 0; c < BN / 32; c++)
                        tma_load_3d(&tm_k, &sm.full[slot], dst + c * C::K_CHUNK, j * BN + c * 32, kh * D, b);
                } else {
#pragma unroll
                    for (int c = 0; c < D / 32; c++)
                        tma_load_3d(&tm_v, &sm.full[slot], dst + c * C::V_CHUNK, kh * D + c * 32, j * BN, b);
                }
                n++;
                return true;
            };
            for (int idx = blockIdx.x; ok && idx < a.n_items; idx += gridDim.x) {
                int b, kh, u;
                item_of(a, idx, b, kh, u);
                const int n_t = item_tiles<NT>(a, u);
                if constexpr (NT == 1) {
                    for (int j = 0; ok && j < C::SBUF && j < n_t; j++) ok = load(true, j, b, kh);
                    for (int j = 0; ok && j < n_t; j++) {
                        ok = load(false, j, b, kh);
                        if (ok && j + C::SBUF < n_t) ok = load(true, j + C::SBUF, b, kh);
                    }
                } else {
                    for (int j = 0; ok && j < n_t; j++) {
                        ok = load(true, j, b, kh);
                        if (ok) ok = load(false, j, b, kh);
                    }
                }
            }
            for (uint32_t i = n > (uint32_t)NS ? n - NS : 0; i < n; i++) mbar_wait_drain(&sm.full[i % NS], (i / NS) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_tf32(BM, BN, false, true);
            constexpr uint32_t idesc_o = idesc_tf32(BM, D, false, true);
            uint32_t n = 0, g = 0;
            int it = 0;
            bool ok = true;
            for (int idx = blockIdx.x; ok && idx < a.n_items; idx += gridDim.x, it++) {
                int b, kh, u;
                item_of(a, idx, b, kh, u);
                const int n_t = item_tiles<NT>(a, u);
                for (int t = 0; ok && t < NT; t++) ok = mbar_wait(&sm.q_full[t], it & 1, err);
                if (!ok) break;
                tc_fence_after();
                if constexpr (NT == 1) {
                    // S(j) = Q K^T(j) into score buffer (g + j) % SBUF
                    auto issue_s = [&](int j) -> bool {
                        const uint32_t s = (g + j) % C::SBUF, slot = n % NS;
                        if (!mbar_wait(&sm.full[slot], (n / NS) & 1, err)) return false;
                        tc_fence_after();
                        const uint32_t k_addr = smem_u32(sm.ring[slot]);
#pragma unroll
                        for (int kk = 0; kk < D / 8; kk++)
                            mma_tf32_ts(tmem + C::S_COL + s * BN, tmem + C::Q_COL + kk * 8,
                                        smem_desc_sw128_32b(k_addr + kk * 1024, C::K_CHUNK, 512), idesc_s, kk > 0 ? 1u : 0u);
                        mma_commit(&sm.empty[slot]);
                        mma_commit(&sm.s_full[0][s]);
                        n++;
                        return true;
                    };
                    for (int j = 0; ok && j < C::SBUF && j < n_t; j++) ok = issue_s(j);
                    for (int j = 0; ok && j < n_t; j++) {
                        const uint32_t gj = g + j, s = gj % C::SBUF;
                        if (!(ok = mbar_wait(&sm.p_full[0][s], (gj / C::SBUF) & 1, err))) break;
                        const uint32_t slot = n % NS;
                        if (!(ok = mbar_wait(&sm.full[slot], (n / NS) & 1, err))) break;
                        tc_fence_after();
                        const uint32_t v_addr = smem_u32(sm.ring[slot]);
#pragma unroll
                        for (int kk = 0; kk < BN / 8; kk++)
                            mma_tf32_ts(tmem + C::O_COL, tmem + C::S_COL + s * BN + kk * 8,
                                        smem_desc_sw128_32b(v_addr + kk * 1024, C::V_CHUNK, 512), idesc_o,
                                        (j > 0 || kk > 0) ? 1u : 0u);
                        mma_commit(&sm.empty[slot]);
                        n++;
                        mma_commit(&sm.pv_done[0][gj & 1]);
                        if (j + C::SBUF < n_t && !(ok = issue_s(j + C::SBUF))) break;
                    }
                } else {
                    // Two query tiles over the ring K0 V0 K1 V1 ...: K(j) is load n0 + 2j,
                    // V(j) load n0 + 2j + 1. Order S_0(0) S_1(0), then per key tile j:
                    // PV_0(j) S_0(j+1) PV_1(j) S_1(j+1). Each tile has one score buffer:
                    // S_t(j+1) overwrites P_t(j) only after PV_t(j) in issue order, and S_t(j)
                    // completes after PV_t(j-1), so the softmax may write P_t(j) and rescale
                    // O_t as soon as it sees S_t(j). A slot is released by its second reader.
                    const uint32_t n0 = n;
                    auto issue_s = [&](int t, int j) -> bool {
                        const uint32_t ln = n0 + 2u * (uint32_t)j, slot = ln % NS;
                        if (t == 0) {
                            if (!mbar_wait(&sm.full[slot], (ln / NS) & 1, err)) return false;
                            tc_fence_after();
                        }
                        const uint32_t k_addr = smem_u32(sm.ring[slot]);
                        const uint32_t tc = (uint32_t)t * C::TILE_COLS;
#pragma unroll
                        for (int kk = 0; kk < D / 8; kk++)
                            mma_tf32_ts(tmem + tc + C::S_COL, tmem + tc + C::Q_COL + kk * 8,
                                        smem_desc_sw128_32b(k_addr + kk * 1024, C::K_CHUNK, 512), idesc_s, kk > 0 ? 1u : 0u);
                        if (t == NT - 1) mma_commit(&sm.empty[slot]);
                        mma_commit(&sm.s_full[t][0]);
                        return true;
                    };
                    for (int t = 0; ok && t < NT && n_t > 0; t++) ok = issue_s(t, 0);
                    for (int j = 0; ok && j < n_t; j++) {
                        const uint32_t gj = g + j;
                        for (int t = 0; ok && t < NT; t++) {
                            if (!(ok = mbar_wait(&sm.p_full[t][0], gj & 1, err))) break;
                            const uint32_t ln = n0 + 2u * (uint32_t)j + 1u, slot = ln % NS;
                            if (t == 0 && !(ok = mbar_wait(&sm.full[slot], (ln / NS) & 1, err))) break;
                            tc_fence_after();
                            const uint32_t v_addr = smem_u32(sm.ring[slot]);
                            const uint32_t tc = (uint32_t)t * C::TILE_COLS;
#pragma unroll
                            for (int kk = 0; kk < BN / 8; kk++)
                                mma_tf32_ts(tmem + tc + C::O_COL, tmem + tc + C::S_COL + kk * 8,
                                            smem_desc_sw128_32b(v_addr + kk * 1024, C::V_CHUNK, 512), idesc_o,
                                            (j > 0 || kk > 0) ? 1u : 0u);
                            if (t == NT - 1) mma_commit(&sm.empty[slot]);
                            mma_commit(&sm.pv_done[t][gj & 1]);
                            if (j + 1 < n_t && !(ok = issue_s(t, j + 1))) break;
                        }
                    }
                    n = n0 + 2u * (uint32_t)n_t;
                }
                g += n_t;
            }
            // every MMA issued so far completes before TMEM is released
            mma_commit(&sm.drain);
            mbar_wait_drain(&sm.drain, 0);
        }
      }
    } else {
        if constexpr (NT == 2) regs_inc<REGS_SOFTMAX>();
        // ------------------------------------------------------------ softmax warpgroups
        const int t = NT == 2 ? (warp - C::SM_WARP0) >> 2 : 0;   // query tile of this warpgroup
        const uint32_t tcol = (uint32_t)t * C::TILE_COLS;        // its TMEM columns
        const int quarter = warp & 3;                  // TMEM lanes this warp may access
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        const float c = 1.4426950408889634f * (D == 64 ? 0.125f : 0.08838834764831845f);  // log2(e)/sqrt(d)
        const int il = row / a.group, hg = row - il * a.group;
        // An item's Q rows into TMEM (zeros for rows past the tile or the chunk). The next
        // item's rows are written as soon as this item's last scores have been seen (its
        // score MMAs, the last readers of Q, are complete), before this item's epilogue, so
        // the next item's first score tiles are computed while the epilogue runs.
        auto load_q = [&](int qidx) {
            int qb, qkh, qu;
            item_of(a, qidx, qb, qkh, qu);
            const int qi = (qu * NT + t) * a.qn + il;     // past n_q for a tile past the last
            const bool qvalid = row < a.rows && qi < a.n_q;
            const float* qrow = a.q + (size_t)qb * a.q_bs + (size_t)(qvalid ? qi : 0) * a.q_stride +
                                (size_t)(qvalid ? qkh * a.group + hg : 0) * D;
#pragma unroll
            for (int cc = 0; cc < D / 32; cc++) {
                uint32_t v[32];
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (qvalid) f = __ldg(reinterpret_cast<const float4*>(qrow + cc * 32 + e));
                    v[e] = __float_as_uint(f.x);
                    v[e + 1] = __float_as_uint(f.y);
                    v[e + 2] = __float_as_uint(f.z);
                    v[e + 3] = __float_as_uint(f.w);
                }
                tmem_st32(tmem + lane_addr + tcol + C::Q_COL + cc * 32, v);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&sm.q_full[t]);
        };
        uint32_t g = 0;
        bool ok = true;
        if ((int)blockIdx.x < a.n_items) load_q(blockIdx.x);
        for (int idx = blockIdx.x; ok && idx < a.n_items; idx += gridDim.x) {
            int b, kh, u;
            item_of(a, idx, b, kh, u);
            const int n_t = item_tiles<NT>(a, u);
            const int mt = u * NT + t;
            const int i = mt * a.qn + il;
            const bool valid = row < a.rows && i < a.n_q;
            const int lim = a.causal ? min(a.n_kv - a.n_q + min(i, a.n_q - 1) + 1, a.n_kv) : a.n_kv;
            float m = 0.f, l = 0.f;
            for (int j = 0; j < n_t; j++) {
                const uint32_t gj = g + j, s = gj % C::SBUF;
                if (!(ok = mbar_wait_warp(&sm.s_full[t][s], (gj / C::SBUF) & 1, err))) break;
                tc_fence_after();
                const uint32_t s_addr = tmem + lane_addr + tcol + C::S_COL + s * BN;
                uint32_t sr[BN];
                tmem_ld128(s_addr, sr);  // the row's 128 scores, one load
                tmem_ld_wait();
                const int valid_keys = lim - j * BN;
                if (valid_keys < BN) {
#pragma unroll
                    for (int e = 0; e < BN; e++)
                        if (e >= valid_keys) sr[e] = __float_as_uint(-INFINITY);
                }
                // row max over 8 independent partial maxima, two new scores per three-input max
                float mx[8];
#pragma unroll
                for (int e = 0; e < 8; e++) mx[e] = fmaxf(__uint_as_float(sr[e]), __uint_as_float(sr[e + 8]));
#pragma unroll
                for (int e0 = 16; e0 < BN; e0 += 16)
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        mx[e] = fmax3(mx[e], __uint_as_float(sr[e0 + e]), __uint_as_float(sr[e0 + 8 + e]));
                const float m_tile =
                    fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], fmax3(mx[5], mx[6], mx[7]))) * c;
                // tile 0 always holds key 0, which every row sees: m_tile is finite there
                float corr = 1.f;
                bool rescale = false;
                if (j == 0) {
                    m = m_tile;
                } else if (m_tile > m + 8.f) {
                    corr = exp2_approx(m - m_tile);
                    m = m_tile;
                    rescale = true;
                }
                float2 ls2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f)};
                const float2 c2 = make_float2(c, c), nm2 = make_float2(-m, -m);
#pragma unroll
                for (int e = 0; e < BN; e += 2) {
                    const float2 x =
                        __ffma2_rn(make_float2(__uint_as_float(sr[e]), __uint_as_float(sr[e + 1])), c2, nm2);
                    const float2 pe = (((e >> 1) & 15) < POLY_PAIRS) ? exp2_poly2(x)
                                                                    : make_float2(exp2_approx(x.x), exp2_approx(x.y));
                    const uint32_t p0 = to_tf32_int(pe.x), p1 = to_tf32_int(pe.y);
                    ls2[(e >> 1) & 3] = __fadd2_rn(ls2[(e >> 1) & 3], make_float2(__uint_as_float(p0), __uint_as_float(p1)));
                    sr[e] = p0;
                    sr[e + 1] = p1;
                }
                {
                    const float2 s01 = __fadd2_rn(ls2[0], ls2[1]), s23 = __fadd2_rn(ls2[2], ls2[3]);
                    const float2 s4 = __fadd2_rn(s01, s23);
                    l = l * corr + (s4.x + s4.y);
                }
                // PV(j - 1) must be done before O is rescaled; without a rescale P(j) is handed
                // to the MMA thread first (its buffer's last reader, PV(j - SBUF), is already
                // done) and the wait comes after, so PV(j) queues behind PV(j - 1) at once.
                // Either way the warp waits for every PV once, in order. PV completions
                // alternate between two barriers: PV(j) may complete before this warp's wait
                // for PV(j - 1) (it needs only the other warps' p_full), and on one barrier
                // that would put the phase two ahead of the parity being waited for; the
                // next completion on PV(j - 1)'s barrier is PV(j + 1), which needs this warp.
                // tcgen05.ld/st are warp-collective: the warp rescales if any of its rows must
                // (corr is 1 in the others).
                const bool any_rescale = __any_sync(0xffffffffu, rescale);
                if (j > 0 && any_rescale) {
                    if (!(ok = mbar_wait_warp(&sm.pv_done[t][(gj - 1) & 1], ((gj - 1) >> 1) & 1, err))) break;
                    tc_fence_after();
                }
                if (any_rescale) {
#pragma unroll
                    for (int cc = 0; cc < D / 32; cc++) {
                        uint32_t o[32];
                        tmem_ld32(tmem + lane_addr + tcol + C::O_COL + cc * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
                        tmem_st32(tmem + lane_addr + tcol + C::O_COL + cc * 32, o);
                    }
                }
                tmem_st128(s_addr, sr);  // P over the scores, one store
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&sm.p_full[t][s]);
                if (j > 0 && !any_rescale) {
                    if (!(ok = mbar_wait_warp(&sm.pv_done[t][(gj - 1) & 1], ((gj - 1) >> 1) & 1, err))) break;
                    tc_fence_after();
                }
            }
            if (!ok) break;
            if (idx + (int)gridDim.x < a.n_items) load_q(idx + gridDim.x);
            // ---- epilogue: O / l -> out[b][i][(kh * group + hg) * D ..]
            const uint32_t g_last = g + n_t - 1;
            if (!(ok = mbar_wait_warp(&sm.pv_done[t][g_last & 1], (g_last >> 1) & 1, err))) break;
            tc_fence_after();
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            float* orow = a.out + (size_t)b * a.out_bs + (size_t)(valid ? i : 0) * a.out_stride +
                          (size_t)(kh * a.group + hg) * D;
#pragma unroll
            for (int cc = 0; cc < D / 32; cc++) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_addr + tcol + C::O_COL + cc * 32, o);
                tmem_ld_wait();
                if (valid) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        const float4 v4 = make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                                                      __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
                        *reinterpret_cast<float4*>(orow + cc * 32 + e) = v4;
                    }
                }
            }
            tc_fence_before();
            g += n_t;
        }
    }

    // warps whose loops ran in lane 0 alone reach the barrier converged
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace prefill_tc

// ---- host side -------------------------------------------------------------------------------

namespace {

bool encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
            const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    return fn(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, int NT>
int launch_kernel(const CUtensorMap& mk, const CUtensorMap& mv, const prefill_tc::Args& a, int grid, cudaStream_t st) {
    using namespace prefill_tc;
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[dev]) {
            if (cudaFuncSetAttribute(prefill_tc_kernel<D, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem_bytes<D, NT>()) != cudaSuccess)
                return -1;
            attr_set[dev] = true;
        }
    }
    prefill_tc_kernel<D, NT><<<grid, Cfg<D, NT>::THREADS, smem_bytes<D, NT>(), st>>>(mk, mv, a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

template <int D>
int launch_d(const FlashParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st) {
    using namespace prefill_tc;
    const int group = (int)(p.n_head / p.n_head_kv);
    const int qn = BM / group;
    Args a{};
    a.out = p.out;
    a.out_stride = p.out_stride;
    a.out_bs = p.out_bs;
    a.n_q = (int)p.n_q;
    a.n_kv = (int)p.n_kv;
    a.n_head_kv = (int)p.n_head_kv;
    a.group = group;
    a.qn = qn;
    a.rows = qn * group;
    a.n_mt = (int)((p.n_q + qn - 1) / qn);
    a.causal = p.causal;
    a.err = err;
    const int slots = sm_count > 0 ? sm_count : 148;
    // d = 64: two query tiles per item unless that leaves a worse last wave. A two-tile item
    // costs about 1.74 one-tile items (measured over config 3's chunks), so the form with
    // fewer item-waves by that weight wins: a full 256-query chunk of 16 sequences (256 pairs
    // = 2 waves against 480 tiles = 4) runs paired, the 208-query last chunk (192 pairs = 2
    // waves against 384 tiles = 3) unpaired.
    const long long per_unit = (long long)n_batch * (long long)p.n_head_kv;
    int nt = 1;
    if (D == 64) {
        const long long w1 = (per_unit * a.n_mt + slots - 1) / slots;
        const long long w2 = (per_unit * ((a.n_mt + 1) / 2) + slots - 1) / slots;
        if (w2 * 174 < w1 * 100) nt = 2;
    }
    a.n_units = (a.n_mt + nt - 1) / nt;
    const long long n_items = per_unit * a.n_units;
    if (n_items <= 0 || n_items >= (1ll << 31)) return -1;
    a.n_items = (int)n_items;

    // a single item: any valid batch stride
    const size_t q_bs = n_batch > 1 ? p.q_bs : p.n_q * p.q_stride;
    const size_t k_bs = n_batch > 1 ? p.k_bs : p.n_head_kv * p.d * p.kt_stride;
    const size_t v_bs = n_batch > 1 ? p.v_bs : p.n_kv * p.kv_stride;
    a.q = p.q;
    a.q_stride = p.q_stride;
    a.q_bs = q_bs;
    CUtensorMap mk, mv;
    {
        cuuint64_t dims[3] = {(cuuint64_t)p.n_kv, (cuuint64_t)(p.n_head_kv * D), (cuuint64_t)n_batch};
        cuuint64_t strides[2] = {(cuuint64_t)p.kt_stride * 4, (cuuint64_t)k_bs * 4};
        cuuint32_t box[3] = {32, (cuuint32_t)D, 1};
        if (!encode(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, p.k, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
            return -1;
    }
    {
        cuuint64_t dims[3] = {(cuuint64_t)(p.n_head_kv * D), (cuuint64_t)p.n_kv, (cuuint64_t)n_batch};
        cuuint64_t strides[2] = {(cuuint64_t)p.kv_stride * 4, (cuuint64_t)v_bs * 4};
        cuuint32_t box[3] = {32, (cuuint32_t)BN, 1};
        if (!encode(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, p.v, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
            return -1;
    }

    const int grid = (int)std::min<long long>(n_items, slots);
    if constexpr (D == 64) {
        if (nt == 2) return launch_kernel<D, 2>(mk, mv, a, grid, st);
    }
    return launch_kernel<D, 1>(mk, mv, a, grid, st);
}

}  // namespace

bool prefill_tc_supported(const FlashParams& p, size_t n_batch) {
    if (!(p.d == 64 || p.d == 128)) return false;
    if (p.kt_stride == 0 || p.n_head_kv == 0 || p.n_head % p.n_head_kv) return false;
    const size_t group = p.n_head / p.n_head_kv;
    if (group == 0 || group > (size_t)prefill_tc::BM) return false;
    if (p.n_q == 0 || p.n_kv == 0 || (p.causal && p.n_kv < p.n_q)) return false;
    if (p.n_q >= (1u << 30) || p.n_kv >= (1u << 30) || n_batch == 0 || n_batch >= (1u << 30)) return false;
    // TMA: 16-byte aligned bases and strides; float4 output stores
    if (((uintptr_t)p.q | (uintptr_t)p.k | (uintptr_t)p.v | (uintptr_t)p.out) & 15) return false;
    if (p.q_stride % 4 || p.kv_stride % 4 || p.kt_stride % 4 || p.out_stride % 4) return false;
    if (n_batch > 1 && (p.q_bs % 4 || p.k_bs % 4 || p.v_bs % 4 || p.out_bs % 4)) return false;
    return true;
}

int prefill_tc_launch(const FlashParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st) {
    if (!prefill_tc_supported(p, n_batch)) return -1;
    return p.d == 64 ? launch_d<64>(p, n_batch, sm_count, err, st) : launch_d<128>(p, n_batch, sm_count, err, st);
}

}  // namespace zwg
