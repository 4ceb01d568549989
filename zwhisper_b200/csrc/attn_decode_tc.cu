// Qwen2 decode attention on tcgen05 tensor cores: one query token per sequence over the
// transposed f32 key cache, kind::tf32 with f32 accumulation, split over the keys.
//
// Reference: the Qwen2 attention call src/llm.zig:191-202 for a decode step (n = 1), which
// runs ops.attentionEx (src/ops.zig:517-541, 562-590) with kt_stride = n_ctx over
// cache_kt[n_head_kv][d][n_ctx] and cache_v[n_ctx][n_head_kv*d]; query head h reads kv head
// h / group (src/ops.zig:521); the single query sees every key.
//
// Why tensor cores for a memory-bound step: the SIMT decode kernel does 4 FLOP per K/V byte
// out of shared memory (every row of a GQA group reads every K and V element), which at
// Qwen2.5-1.5B batch sizes costs more than streaming the bytes. Here the group's rows are
// the M side of the MMA: a 128-row tile holds the `group` query heads of one kv head in rows
// 0..group-1 (the rest are zero), so the tensor pipe does the arithmetic at a small fraction
// of its rate and the kernel is bound by the K/V stream again.
//
// Design (the operand layouts and the MMA/softmax hand-off of the tf32 prefill kernel):
//   - Work: a segment is one (sequence, kv head); its keys are cut into `pieces` equal
//     ranges of 64-key tiles, one per CTA. A CTA with the whole segment writes the output;
//     otherwise it writes a partial (max, sum, unnormalised O) per row and the last CTA of
//     the segment (atomic ticket, reset by that CTA) merges them with all its threads.
//   - Q lives in TMEM, not shared memory: the softmax warp writes the group's rows (tf32,
//     rows >= group zero) with tcgen05.st and S = Q K^T takes its A operand from TMEM, as
//     O += P V does. The 64 KB a 128-row Q tile would take in shared memory go to the K/V
//     rings instead: three stages each, so a CTA has three tiles of loads ahead of its
//     MMAs (with two, every tile waited a whole load latency: ~1.3 us per tile).
//   - K^T tiles: two [d][32 keys] boxes, the MN-major B operand of S = Q K^T; V tiles:
//     [64 keys][32 columns] boxes, the MN-major B operand of O += P V (both in the 128-byte
//     swizzle with 32-byte atoms, descriptor layout 1).
//   - TMEM: two 64-column score buffers (P written back over S as tf32, the TMEM A operand
//     of the PV MMA), a d-column O accumulator and the d-column Q.
//   - Warp 0: TMA producers (lane 0: K^T, lane 1: V). Warp 1: TMEM allocation and the MMA
//     thread (S0 S1 | PV0 S2 | PV1 S3 ...). Warp 4 (TMEM lanes 0..31): Q into TMEM, then the
//     softmax of the group's rows, one thread per row, online max in base 2 kept stale
//     unless it grows by more than 2^8, P rounded to tf32. Warps 2, 3 and 5 only join the
//     merge. (Spreading the softmax over four warps, one per lane quarter with a copy of Q
//     each, measured slower: at batch the kernel is at the DRAM stream's pace after the
//     first tile, and the extra combine only adds.)
// Every wait is bounded; a wait that runs out records kErrTimeout, the CTA drains its own
// copies and MMAs with bounded waits, frees TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "chain.cuh"
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace zwg {
namespace decode_tc {

using namespace sm100;

constexpr int BM = 128;                // rows per tile = TMEM lanes
constexpr int BN = 64;                 // keys per tile
constexpr int THREADS = 192;           // warp 0 TMA, warp 1 MMA, warp 4 softmax, all merge
constexpr int NST = 3;                 // K and V ring stages
constexpr uint32_t O_COL = 2 * BN;     // S/P buffers 2 x 64 columns, then O, then Q
constexpr int MAX_PIECES = 16;         // pieces per segment the workspace holds
constexpr int PM = 8;                  // pieces merged per batch of loads

template <int D>
struct Cfg {
    static constexpr uint32_t K_CHUNK = D * 128;            // [D rows][32 keys]
    static constexpr uint32_t K_BYTES = 2 * K_CHUNK;
    static constexpr uint32_t V_CHUNK = BN * 128;           // [64 keys][32 floats]
    static constexpr uint32_t V_BYTES = (D / 32) * V_CHUNK;
    static constexpr uint32_t Q_COL = O_COL + D;
    static constexpr uint32_t TMEM_COLS = D == 128 ? 512 : 256;  // a power of two >= 2 * 64 + 2 * D
    // d = 64: 96 KB of rings, two CTAs per SM; d = 128: 192 KB, one
    static constexpr int CTAS_PER_SM = D == 64 ? 2 : 1;
};

template <int D>
struct Smem {
    alignas(1024) uint8_t k[NST][Cfg<D>::K_BYTES];
    alignas(1024) uint8_t v[NST][Cfg<D>::V_BYTES];
    uint64_t q_full;
    uint64_t k_full[NST], k_empty[NST], v_full[NST], v_empty[NST];
    uint64_t s_full[2], p_full[2], pv_done[2], drain;
    uint32_t tmem_base;
    int abort_flag;
    int last;
};

template <int D>
constexpr size_t smem_bytes() {
    return sizeof(Smem<D>) + 1024;  // + alignment slack
}

struct Args {
    const float* q;  // [batch][1][n_head * D] at q_bs per item
    size_t q_bs;
    float* out;
    size_t out_stride, out_bs;
    int n_kv, n_head_kv, group, n_t, pieces, n_items;
    float* part;    // [segment][MAX_PIECES][group][D + 2]: max, sum, O
    int* counters;  // [segment] tickets, zero between calls
    int* err;
};

template <int D>
__global__ void __launch_bounds__(THREADS, Cfg<D>::CTAS_PER_SM)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const Args a) {
    using C = Cfg<D>;
    extern __shared__ uint8_t smem_raw[];
    Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int* err = a.err;

    const int idx = blockIdx.x;
    const int seg = idx / a.pieces, piece = idx - seg * a.pieces;
    const int b = seg / a.n_head_kv, kh = seg - b * a.n_head_kv;
    const int t_first = (int)(((long long)piece * a.n_t) / a.pieces);
    const int n_t = (int)(((long long)(piece + 1) * a.n_t) / a.pieces) - t_first;

    // launched as a programmatic dependent of the kernel before it (the q/k/v projection of
    // a decode step): the next kernel may start as soon as every CTA got here
    chain_release();
    if (threadIdx.x == 0) {
        sm.abort_flag = err ? *(volatile int*)err : 0;
        sm.last = 0;
    }
    __syncthreads();
    if (sm.abort_flag || n_t <= 0) return;

    if (threadIdx.x == 0) {
        mbar_init(&sm.q_full, 32);
        for (int s = 0; s < NST; s++) {
            mbar_init(&sm.k_full[s], 1);
            mbar_init(&sm.k_empty[s], 1);
            mbar_init(&sm.v_full[s], 1);
            mbar_init(&sm.v_empty[s], 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&sm.s_full[s], 1);
            mbar_init(&sm.p_full[s], 32);
        }
        mbar_init(&sm.pv_done[0], 1);
        mbar_init(&sm.pv_done[1], 1);
        mbar_init(&sm.drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&sm.tmem_base, C::TMEM_COLS);
        tmem_relinquish();
    }
    // While the previous kernel finishes: the first K^T and V tiles of this piece into L2 (a
    // prefetch reads nothing into the CTA, so data the previous kernel is still writing is
    // read only after the wait below, from the coherent L2). Then every thread waits for the
    // previous kernel before any read of q, K, V or the workspace and any write.
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        const int n_pre = n_t < NST + 1 ? n_t : NST + 1;
        for (int j = 0; j < n_pre; j++) {
            const int key0 = (t_first + j) * BN;
            tma_prefetch_3d(&tm_k, key0, kh * D, b);
            tma_prefetch_3d(&tm_k, key0 + 32, kh * D, b);
            for (int c = 0; c < D / 32; c++) tma_prefetch_3d(&tm_v, kh * D + c * 32, key0, b);
        }
    }
    chain_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const float c_log2 = 1.4426950408889634f * (D == 64 ? 0.125f : 0.08838834764831845f);  // log2(e)/sqrt(d)
    float m = 0.f, l = 0.f;  // softmax state of row `lane` (warp 4)

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producers
        // Each lane waits at exit for the last load it issued, so no copy is in flight when
        // the CTA releases its memory.
        if (lane == 0) {
            prefetch_tmap(&tm_k);
            uint32_t n_k_loads = 0;
            bool ok = true;
            for (int j = 0; ok && j < n_t; j++) {
                const uint32_t s = j % NST;
                if (j >= NST && !(ok = mbar_wait(&sm.k_empty[s], ((j / NST) - 1) & 1, err))) break;
                const int key0 = (t_first + j) * BN;
                mbar_arrive_expect_tx(&sm.k_full[s], C::K_BYTES);
                tma_load_3d(&tm_k, &sm.k_full[s], sm.k[s], key0, kh * D, b);
                tma_load_3d(&tm_k, &sm.k_full[s], sm.k[s] + C::K_CHUNK, key0 + 32, kh * D, b);
                n_k_loads++;
            }
            // the last load of each stage: stage st took loads st, st + NST, ...
            for (uint32_t st = 0; st < NST && st < n_k_loads; st++)
                mbar_wait_drain(&sm.k_full[st], ((n_k_loads - 1 - st) / NST) & 1);
        } else if (lane == 1) {
            prefetch_tmap(&tm_v);
            uint32_t n_v_loads = 0;
            bool ok = true;
            for (int j = 0; ok && j < n_t; j++) {
                const uint32_t s = j % NST;
                if (j >= NST && !(ok = mbar_wait(&sm.v_empty[s], ((j / NST) - 1) & 1, err))) break;
                const int key0 = (t_first + j) * BN;
                mbar_arrive_expect_tx(&sm.v_full[s], C::V_BYTES);
                for (int c = 0; c < D / 32; c++)
                    tma_load_3d(&tm_v, &sm.v_full[s], sm.v[s] + c * C::V_CHUNK, kh * D + c * 32, key0, b);
                n_v_loads++;
            }
            for (uint32_t st = 0; st < NST && st < n_v_loads; st++)
                mbar_wait_drain(&sm.v_full[st], ((n_v_loads - 1 - st) / NST) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_tf32(BM, BN, false, true);
            constexpr uint32_t idesc_o = idesc_tf32(BM, D, false, true);
            bool ok = mbar_wait(&sm.q_full, 0, err);
            tc_fence_after();
            // S(j) = Q K^T(j) into score buffer j % 2, Q from TMEM
            auto issue_s = [&](int j) -> bool {
                const uint32_t st = j % NST, s = j & 1;
                if (!mbar_wait(&sm.k_full[st], (j / NST) & 1, err)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sm.k[st]);
#pragma unroll
                for (int kk = 0; kk < D / 8; kk++) {
                    const uint64_t bd = smem_desc_sw128_32b(k_addr + kk * 1024, C::K_CHUNK, 512);
                    mma_tf32_ts(tmem + s * BN, tmem + C::Q_COL + kk * 8, bd, idesc_s, kk > 0 ? 1u : 0u);
                }
                mma_commit(&sm.k_empty[st]);
                mma_commit(&sm.s_full[s]);
                return true;
            };
            if (ok) ok = issue_s(0);
            if (ok && n_t > 1) ok = issue_s(1);
            for (int j = 0; ok && j < n_t; j++) {
                const uint32_t st = j % NST, s = j & 1;
                if (!(ok = mbar_wait(&sm.p_full[s], (j >> 1) & 1, err))) break;
                if (!(ok = mbar_wait(&sm.v_full[st], (j / NST) & 1, err))) break;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sm.v[st]);
#pragma unroll
                for (int kk = 0; kk < BN / 8; kk++) {
                    const uint64_t bd = smem_desc_sw128_32b(v_addr + kk * 1024, C::V_CHUNK, 512);
                    mma_tf32_ts(tmem + O_COL, tmem + s * BN + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&sm.pv_done[j & 1]);
                mma_commit(&sm.v_empty[st]);
                if (j + 2 < n_t && !(ok = issue_s(j + 2))) break;
            }
            // every MMA issued so far completes before TMEM is released
            mma_commit(&sm.drain);
            mbar_wait_drain(&sm.drain, 0);
        }
    } else if (warp == 4) {
        // ------------------------------------------------------------ softmax, rows 0..31
        // (a warp reaches the TMEM lanes of its index mod 4: warp 4 has lanes 0..31)
        const int row = lane;
        const bool valid = row < a.group;
        // Q rows of the group into TMEM lanes 0..31 as tf32 (rows >= group zero)
        {
            const float4* qrow = reinterpret_cast<const float4*>(
                a.q + (size_t)b * a.q_bs + (size_t)(kh * a.group + (valid ? row : 0)) * D);
#pragma unroll
            for (int cc = 0; cc < D / 32; cc++) {
                uint32_t r[32];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float4 f = valid ? __ldg(qrow + cc * 8 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
                    r[4 * e] = to_tf32_int(f.x);
                    r[4 * e + 1] = to_tf32_int(f.y);
                    r[4 * e + 2] = to_tf32_int(f.z);
                    r[4 * e + 3] = to_tf32_int(f.w);
                }
                tmem_st32(tmem + C::Q_COL + cc * 32, r);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&sm.q_full);
        }
        bool ok = true;
        for (int j = 0; j < n_t; j++) {
            const uint32_t s = j & 1;
            if (!(ok = mbar_wait_warp(&sm.s_full[s], (j >> 1) & 1, err))) break;
            tc_fence_after();
            const uint32_t s_addr = tmem + s * BN;  // lanes 0..31: this warp's quarter
            uint32_t sr[64];
            {
                uint32_t x[32], y[32];
                tmem_ld32(s_addr, x);
                tmem_ld32(s_addr + 32, y);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    sr[e] = x[e];
                    sr[32 + e] = y[e];
                }
            }
            const int valid_keys = a.n_kv - (t_first + j) * BN;
            if (valid_keys < BN) {
#pragma unroll
                for (int e = 0; e < 64; e++)
                    if (e >= valid_keys) sr[e] = __float_as_uint(-INFINITY);
            }
            float mx[8];
#pragma unroll
            for (int e = 0; e < 8; e++) mx[e] = __uint_as_float(sr[e]);
#pragma unroll
            for (int e = 8; e < 64; e++) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(sr[e]));
#pragma unroll
            for (int e = 0; e < 4; e++) mx[e] = fmaxf(mx[e], mx[e + 4]);
            // every tile of a piece holds at least one key below n_kv: m_tile is finite
            const float m_tile = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * c_log2;
            float corr = 1.f;
            bool rescale = false;
            if (j == 0) {
                m = m_tile;
            } else if (m_tile > m + 8.f) {
                corr = exp2_approx(m - m_tile);
                m = m_tile;
                rescale = true;
            }
            float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int e = 0; e < 64; e++) {
                const uint32_t p = to_tf32_int(exp2_approx(fmaf(__uint_as_float(sr[e]), c_log2, -m)));
                ls[e & 3] += __uint_as_float(p);
                sr[e] = p;
            }
            l = l * corr + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
            // PV(j - 1) must be done before O is rescaled; without a rescale P(j) is handed to
            // the MMA thread first (its buffer's last reader, PV(j - 2), is already done) and
            // the wait comes after, so PV(j) queues behind PV(j - 1) at once. Either way the
            // warp waits for every PV once, in order. PV completions alternate between two
            // barriers, so PV(j) completing before the wait for PV(j - 1) cannot put that
            // barrier's phase two ahead of the parity waited for.
            // tcgen05.ld/st are warp-collective: the warp rescales if any of its rows must.
            const bool any_rescale = __any_sync(0xffffffffu, rescale);
            if (j > 0 && any_rescale) {
                if (!(ok = mbar_wait_warp(&sm.pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err))) break;
                tc_fence_after();
#pragma unroll
                for (int cc = 0; cc < D / 32; cc++) {
                    uint32_t o[32];
                    tmem_ld32(tmem + O_COL + cc * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
                    tmem_st32(tmem + O_COL + cc * 32, o);
                }
            }
            {
                uint32_t x[32], y[32];
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    x[e] = sr[e];
                    y[e] = sr[32 + e];
                }
                tmem_st32(s_addr, x);
                tmem_st32(s_addr + 32, y);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&sm.p_full[s]);
            if (j > 0 && !any_rescale) {
                if (!(ok = mbar_wait_warp(&sm.pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err))) break;
                tc_fence_after();
            }
        }
        if (ok) ok = mbar_wait_warp(&sm.pv_done[(n_t - 1) & 1], ((n_t - 1) >> 1) & 1, err);
        if (ok) {
            // ---- epilogue: the output (one piece) or this piece's partial
            tc_fence_after();
            const bool whole = a.pieces == 1;
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            float* orow = a.out + (size_t)b * a.out_bs + (size_t)(kh * a.group + (valid ? row : 0)) * D;
            float* prow = a.part + (((size_t)seg * MAX_PIECES + piece) * a.group + (valid ? row : 0)) * (D + 2);
#pragma unroll
            for (int cc = 0; cc < D / 32; cc++) {
                uint32_t o[32];
                tmem_ld32(tmem + O_COL + cc * 32, o);
                tmem_ld_wait();
                if (valid) {
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        const float v = __uint_as_float(o[e]);
                        if (whole) orow[cc * 32 + e] = v * inv;
                        else prow[2 + cc * 32 + e] = v;
                    }
                }
            }
            if (!whole) {
                if (valid) {
                    prow[0] = m;
                    prow[1] = l;
                }
                // the last CTA of the segment merges: every lane's fence orders its partial
                // before the ticket
                __threadfence();
                __syncwarp();
                if (lane == 0) {
                    const int done = atomicAdd(&a.counters[seg], 1);
                    if (done == a.pieces - 1) {
                        a.counters[seg] = 0;  // ready for the next call
                        sm.last = 1;
                    }
                    __threadfence();
                }
            }
        } else if (lane == 0) {
            *(volatile int*)&sm.abort_flag = 1;
        }
        tc_fence_before();
    }

    // warps whose loops ran in lane 0 alone reach the barrier converged
    __syncwarp();
    __syncthreads();
    if (sm.last && !*(volatile int*)&sm.abort_flag) {
        // ---- merge of the segment's pieces: thread = (row, 4 columns)
        constexpr int C4 = D / 4;
        for (int it = threadIdx.x; it < a.group * C4; it += THREADS) {
            const int r = it / C4, c4 = it - r * C4;
            float M = -INFINITY, L = 0.f;
            float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p0 = 0; p0 < a.pieces; p0 += PM) {
                float mp[PM], lp[PM];
                float4 op[PM];
#pragma unroll
                for (int u = 0; u < PM; u++) {
                    mp[u] = -INFINITY;
                    lp[u] = 0.f;
                    op[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (p0 + u < a.pieces) {
                        const float* pr = a.part + (((size_t)seg * MAX_PIECES + p0 + u) * a.group + r) * (D + 2);
                        mp[u] = __ldcg(pr);
                        lp[u] = __ldcg(pr + 1);
                        const float* po = pr + 2 + 4 * c4;
                        op[u] = make_float4(__ldcg(po), __ldcg(po + 1), __ldcg(po + 2), __ldcg(po + 3));
                    }
                }
                float Mn = M;
#pragma unroll
                for (int u = 0; u < PM; u++) Mn = fmaxf(Mn, mp[u]);
                const float cm = M == -INFINITY ? 0.f : exp2_approx(M - Mn);
                L *= cm;
                O.x *= cm; O.y *= cm; O.z *= cm; O.w *= cm;
#pragma unroll
                for (int u = 0; u < PM; u++) {
                    const float ew = mp[u] == -INFINITY ? 0.f : exp2_approx(mp[u] - Mn);
                    L += lp[u] * ew;
                    O.x += op[u].x * ew; O.y += op[u].y * ew; O.z += op[u].z * ew; O.w += op[u].w * ew;
                }
                M = Mn;
            }
            const float inv = L > 0.f ? 1.0f / L : 0.f;
            float* orow = a.out + (size_t)b * a.out_bs + (size_t)(kh * a.group + r) * D + 4 * c4;
            orow[0] = O.x * inv;
            orow[1] = O.y * inv;
            orow[2] = O.z * inv;
            orow[3] = O.w * inv;
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace decode_tc

// ---- host side -------------------------------------------------------------------------------

namespace {

bool encode_map(CUtensorMap* m, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes, box,
              es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Pieces per segment: enough CTAs to fill the SMs' slots once, at most one per tile and at
// most MAX_PIECES.
int pieces_for(size_t segs, int n_t, int d, int sm_count) {
    const long long slots = (long long)std::max(1, sm_count) * (d == 64 ? 2 : 1);
    long long p = slots / (long long)std::max<size_t>(1, segs);
    p = std::min<long long>(p, n_t);
    p = std::min<long long>(p, decode_tc::MAX_PIECES);
    return (int)std::max<long long>(1, p);
}

template <int D>
int launch_d(const DecodeParams& p, size_t n_batch, int sm_count, cudaStream_t st, int* err) {
    using namespace decode_tc;
    Args a{};
    a.q = p.q;
    a.q_bs = n_batch > 1 ? p.q_bs : 0;
    a.out = p.out;
    a.out_stride = p.out_stride;
    a.out_bs = p.out_bs;
    a.n_kv = (int)p.n_kv;
    a.n_head_kv = (int)p.n_head_kv;
    a.group = (int)(p.n_head / p.n_head_kv);
    a.n_t = (int)((p.n_kv + BN - 1) / BN);
    const size_t segs = n_batch * p.n_head_kv;
    a.pieces = pieces_for(segs, a.n_t, D, sm_count);
    const long long n_items = (long long)segs * a.pieces;
    if (n_items <= 0 || n_items >= (1ll << 31)) return -1;
    a.n_items = (int)n_items;
    a.part = p.ws;
    const size_t parts = segs * MAX_PIECES * (size_t)a.group * (D + 2) * sizeof(float);
    a.err = err;
    if (p.tickets) {
        a.counters = p.tickets;
    } else {
        a.counters = reinterpret_cast<int*>(reinterpret_cast<char*>(p.ws) + ((parts + 255) / 256) * 256);
        if (a.pieces > 1 && cudaMemsetAsync(a.counters, 0, segs * sizeof(int), st) != cudaSuccess) return -1;
    }

    // a single item: any valid batch stride
    const size_t k_bs = n_batch > 1 ? p.k_bs : p.n_head_kv * D * p.kt_stride;
    const size_t v_bs = n_batch > 1 ? p.v_bs : p.n_kv * p.kv_stride;
    CUtensorMap mk, mv;
    {
        cuuint64_t dims[3] = {(cuuint64_t)p.n_kv, (cuuint64_t)(p.n_head_kv * D), (cuuint64_t)n_batch};
        cuuint64_t strides[2] = {(cuuint64_t)p.kt_stride * 4, (cuuint64_t)k_bs * 4};
        cuuint32_t box[3] = {32, (cuuint32_t)D, 1};
        if (!encode_map(&mk, 3, p.k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) return -1;
    }
    {
        cuuint64_t dims[3] = {(cuuint64_t)(p.n_head_kv * D), (cuuint64_t)p.n_kv, (cuuint64_t)n_batch};
        cuuint64_t strides[2] = {(cuuint64_t)p.kv_stride * 4, (cuuint64_t)v_bs * 4};
        cuuint32_t box[3] = {32, (cuuint32_t)BN, 1};
        if (!encode_map(&mv, 3, p.v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) return -1;
    }

    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[dev]) {
            if (cudaFuncSetAttribute(decode_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem_bytes<D>()) != cudaSuccess)
                return -1;
            attr_set[dev] = true;
        }
    }
    if (launch_chained_smem(decode_tc_kernel<D>, dim3(a.n_items), dim3(THREADS), smem_bytes<D>(), st, mk, mv, a) !=
        cudaSuccess)
        return -1;
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace

bool decode_tc_supported(const DecodeParams& p, size_t n_batch) {
    if (!(p.d == 64 || p.d == 128)) return false;
    if (p.n_q != 1 || p.kt_stride == 0 || p.n_head_kv == 0 || p.n_head % p.n_head_kv) return false;
    const size_t group = p.n_head / p.n_head_kv;
    if (group == 0 || group > 32) return false;  // the group's rows are the softmax warp's lanes
    if (p.n_kv == 0 || p.n_kv >= (1u << 30) || n_batch == 0 || n_batch >= (1u << 30)) return false;
    // TMA: 16-byte aligned bases and strides
    if (((uintptr_t)p.q | (uintptr_t)p.k | (uintptr_t)p.v) & 15) return false;
    if (((uintptr_t)p.out) & 3) return false;
    if (p.q_stride % 4 || p.kv_stride % 4 || p.kt_stride % 4) return false;
    if (n_batch > 1 && (p.q_bs % 4 || p.k_bs % 4 || p.v_bs % 4)) return false;
    return true;
}

size_t decode_tc_workspace_bytes(size_t n_batch, size_t n_head_kv, size_t group, size_t d) {
    const size_t segs = n_batch * n_head_kv;
    const size_t parts = segs * decode_tc::MAX_PIECES * group * (d + 2) * sizeof(float);
    return ((parts + 255) / 256) * 256 + segs * sizeof(int);
}

int decode_tc_launch(const DecodeParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st) {
    if (!decode_tc_supported(p, n_batch)) return -1;
    return p.d == 64 ? launch_d<64>(p, n_batch, sm_count, st, err) : launch_d<128>(p, n_batch, sm_count, st, err);
}

}  // namespace zwg
