// Decode attention fed by TMA, stream-K scheduled (sm_100a): the memory-bound single-token
// steps of the decoder (self- and cross-attention, src/decoder.zig:184 and :191) and of
// Qwen2 over its transposed key cache (src/llm.zig:191-202).
//
// Work space: a segment is one (item, kv head) pair; its keys are split into tiles of 32.
// All R = n_q * group query rows that read a kv head are processed together, so each K/V
// byte is read once per GQA group. The segments' tiles are laid end to end and every CTA of
// a persistent grid takes an equal contiguous range of them (stream-K): no wave
// quantization, whatever the batch (with at least as many segments as CTAs, ranges hold
// whole segments instead). A range can start or end inside a segment; each CTA
// merges what it computed for a segment into one partial (max, sum, accumulator), and the
// last CTA to finish a segment (atomic ticket) merges that segment's pieces and writes the
// output; a segment held by one CTA is written directly.
//   warp NW     producers: lane 1 loads each segment's q rows (bulk copy into one of two q
//               buffers, a segment ahead); lane 0 loads the K and V tiles of 32 keys into an
//               NS-slot ring
//               with 3-D TMA tile loads (no multicast): K^T boxes [d][32] for the transposed
//               cache, row boxes [32][d] otherwise, V boxes [32][d]; 192 KB of ring, so a team's
//               next tiles are loading while it computes the current one.
//   compute warps, in teams of up to 4 warps that share a tile and split its query
//               rows (a GQA group's 6-8 rows spread over 4 warps); team t takes the range's
//               tiles t, t + NT, ... (ring slot = tile % NS): scores with one lane per key,
//               online softmax in base 2 per warp (warp max, lane-partial sums),
//               probabilities through shared memory, P.V with D/4 lanes per value row; at a
//               segment's end the teams merge in shared memory.
// Keys past n_kv are masked to -inf per row, with the causal limit n_kv - n_q + i + 1 of
// query row i (src/ops.zig:534).
//
// Every mbarrier wait is bounded (sm100::mbar_wait); a timeout records kErrTimeout in the
// error word and the CTA leaves.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <set>

#include "chain.cuh"
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace zwg {

using namespace sm100;

namespace dec_tma {

constexpr int TK = 32;  // keys per tile

// Warps per tile (a team): the query rows are split over the team, up to 4 warps with
// RMAX / 4 rows each, so the per-key work of a GQA group spreads over several warps.
// Ring slots belong to teams: slot = tile % NS and team = tile % NT with NS a multiple of
// NT, so each slot is only ever filled for, and released by, one team, and a team's parity
// waits on its slots cannot alias a fill meant for another team.
template <int D, int RMAX>
struct Cfg {
    static constexpr int NS_MAX = D >= 128 ? 6 : D >= 64 ? 12 : 16;  // 192 KB of ring at most
    static constexpr int NWR = RMAX >= 4 ? 4 : RMAX;                  // warps per team
    static constexpr int RPW = RMAX / NWR;                            // rows per warp
    // up to 12 compute warps: three teams of four for GQA groups (more tiles in flight per
    // CTA than two teams: 6-12% faster on the Qwen2 shapes; four teams gained nothing more)
    static constexpr int NT = (12 / NWR) < (NS_MAX / 2) ? (12 / NWR) : (NS_MAX / 2);  // teams
    static constexpr int NS = NT * (NS_MAX / NT);                     // ring slots
    static constexpr int NW = NT * NWR;                               // compute warps
    static constexpr int THREADS = (NW + 1) * 32;
    static constexpr uint32_t TILE_BYTES = TK * D * 4;
    static constexpr int LPK = D / 4;                                 // lanes per value row (P.V)
    static constexpr int KPS = 32 / LPK;                              // value rows per warp step
    static_assert(NS % NT == 0 && NS >= 2 * NT, "every team owns at least two ring slots");
};

template <int D, int RMAX>
struct Smem {
    using C = Cfg<D, RMAX>;
    float k[C::NS][TK * D];           // K^T: [D][32]; rows: [32][D]
    float v[C::NS][TK * D];           // [32][D]
    float q[2][RMAX][D];              // row r = qi * G + g (rows >= R are never read unmasked)
    float p[C::NW][C::RPW][TK];
    float mo[C::NT][RMAX][D];         // merge over teams: accumulators
    float mm[C::NT][RMAX];            // maxima
    float ml[C::NT][RMAX];            // sums
    uint64_t full[C::NS], empty[C::NS];
    uint64_t q_full[2], q_empty[2];
    int last;                         // this CTA completes the segment's merge
    int abort_flag;
};

template <int D, int RMAX>
constexpr size_t smem_bytes() {
    return sizeof(Smem<D, RMAX>) + 128;
}
static_assert(sizeof(Smem<128, 8>) + 128 <= 227 * 1024, "shared memory over the per-block limit");
static_assert(sizeof(Smem<128, 1>) + 128 <= 227 * 1024, "shared memory over the per-block limit");
static_assert(sizeof(Smem<64, 8>) + 128 <= 227 * 1024, "shared memory over the per-block limit");
static_assert(sizeof(Smem<64, 1>) + 128 <= 227 * 1024, "shared memory over the per-block limit");
static_assert(sizeof(Smem<32, 8>) + 128 <= 227 * 1024, "shared memory over the per-block limit");

struct Geo {
    long long total;  // tiles of all segments
    int n_t;          // tiles per segment
    int n_segs;
    int p_max;        // pieces per segment the workspace holds
    int mode;         // 0: equal ranges over all tiles (stream-K); 1: whole segments per CTA
                      // (at least as many segments as CTAs); 2: every segment cut into
                      // `pieces` equal pieces, one per CTA (few segments, many CTAs)
    int pieces;
};

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// First tile of CTA c, for G CTAs over the T tiles of `geo`: equal ranges; or, with at least
// as many segments as CTAs, equal numbers of whole segments (no segment is then shared, and
// no CTA pays the merge of a shared segment); or, with many more CTAs than segments, one
// piece of one segment per CTA (no CTA holds two segments, so each pays one merge).
__host__ __device__ __forceinline__ long long range_begin(long long c, const Geo& geo, long long G) {
    if (geo.mode == 1) return (c * geo.n_segs / G) * geo.n_t;
    if (geo.mode == 2) {
        if (c >= (long long)geo.n_segs * geo.pieces) return geo.total;
        const long long seg = c / geo.pieces, pc = c % geo.pieces;
        return seg * geo.n_t + (pc * geo.n_t) / geo.pieces;
    }
    return c * geo.total / G;
}
// The CTA whose range holds tile x.
__host__ __device__ __forceinline__ int owner_of(long long x, const Geo& geo, int G) {
    long long c = x * G / geo.total;
    while (c + 1 < G && range_begin(c + 1, geo, G) <= x) c++;
    while (c > 0 && range_begin(c, geo, G) > x) c--;
    return (int)c;
}

template <int D, bool KT, int RMAX>
__global__ void __launch_bounds__(Cfg<D, RMAX>::THREADS, 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      DecodeParams p, Geo geo, int* counters, int* err) {
    using C = Cfg<D, RMAX>;
    extern __shared__ uint8_t smem_raw[];
    Smem<D, RMAX>& sm = *reinterpret_cast<Smem<D, RMAX>*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = (int)(p.n_head / p.n_head_kv);
    const int R = (int)p.n_q * G;
    const int n_kv = (int)p.n_kv;
    const long long t_begin = range_begin(blockIdx.x, geo, gridDim.x);
    const long long t_end = range_begin(blockIdx.x + 1, geo, gridDim.x);

    // launched as a programmatic dependent of the kernel before it (the q/k/v projection of
    // a decode step): the next kernel may start as soon as every CTA got here
    chain_release();
    if (threadIdx.x == 0) sm.abort_flag = err ? *(volatile int*)err : 0;
    __syncthreads();
    if (sm.abort_flag || t_begin >= t_end) return;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NS; s++) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], C::NWR);  // every warp of the team releases
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&sm.q_full[b], 1);
            mbar_init(&sm.q_empty[b], 1);
        }
        fence_mbar_init();
    }
    // While the previous kernel finishes: this CTA's first K and V tiles into L2 (a prefetch
    // reads nothing into the CTA, so data the previous kernel is still writing is read only
    // after the wait, from the coherent L2). Then every thread waits for the previous kernel
    // before any read of q, K, V or the workspace and any write.
    if (warp == C::NW && lane == 0) {
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        const long long x_end = std::min<long long>(t_end, t_begin + C::NS);
        for (long long x = t_begin; x < x_end; x++) {
            const int seg = (int)(x / geo.n_t);
            const int hk = seg % (int)p.n_head_kv;
            const int b = seg / (int)p.n_head_kv;
            const int t0 = (int)(x - (long long)seg * geo.n_t) * TK;
            if (KT) tma_prefetch_3d(&tm_k, t0, hk * D, b);
            else tma_prefetch_3d(&tm_k, hk * D, t0, b);
            tma_prefetch_3d(&tm_v, hk * D, t0, b);
        }
    }
    chain_wait();
    __syncthreads();

    if (warp == C::NW) {
        // ---------------------------------------------------------------- producers
        if (lane == 1) {
            // q rows of each segment, one buffer ahead of the compute warps
            bool ok = true;
            long long x = t_begin;
            for (int si = 0; ok && x < t_end; si++) {
                const int seg = (int)(x / geo.n_t);
                const int hk = seg % (int)p.n_head_kv;
                const int b = seg / (int)p.n_head_kv;
                const int qb = si & 1;
                if (si >= 2 && !(ok = mbar_wait(&sm.q_empty[qb], ((si >> 1) - 1) & 1, err))) break;
                mbar_arrive_expect_tx(&sm.q_full[qb], (uint32_t)(p.n_q * G * D * 4));
                for (int qi = 0; qi < (int)p.n_q; qi++)
                    bulk_load(&sm.q[qb][qi * G][0], p.q + (size_t)b * p.q_bs + (size_t)qi * p.q_stride + (size_t)hk * G * D,
                              (uint32_t)(G * D * 4), &sm.q_full[qb]);
                x = std::min<long long>(t_end, (long long)(seg + 1) * geo.n_t);
            }
        } else if (lane == 0) {
            // K and V tiles
            prefetch_tmap(&tm_k);
            prefetch_tmap(&tm_v);
            bool ok = true;
            long long x = t_begin;
            for (int si = 0; ok && x < t_end; si++) {
                const int seg = (int)(x / geo.n_t);
                const long long seg_end = std::min<long long>(t_end, (long long)(seg + 1) * geo.n_t);
                const int hk = seg % (int)p.n_head_kv;
                const int b = seg / (int)p.n_head_kv;
                for (; x < seg_end; x++) {
                    const long long i = x - t_begin;      // local tile index
                    const int s = (int)(i % C::NS);
                    if (i >= C::NS && !(ok = mbar_wait(&sm.empty[s], (uint32_t)((i / C::NS) - 1) & 1, err))) break;
                    const int t0 = (int)(x - (long long)seg * geo.n_t) * TK;
                    mbar_arrive_expect_tx(&sm.full[s], 2 * C::TILE_BYTES);
                    if (KT) tma_load_3d(&tm_k, &sm.full[s], sm.k[s], t0, hk * D, b);
                    else tma_load_3d(&tm_k, &sm.full[s], sm.k[s], hk * D, t0, b);
                    tma_load_3d(&tm_v, &sm.full[s], sm.v[s], hk * D, t0, b);
                }
            }
        }
        return;
    }

    // -------------------------------------------------------------------- compute warps
    constexpr int NWR = C::NWR, RPW = C::RPW, NT = C::NT;
    const int team = warp / NWR;           // which tiles: local tile i with i % NT == team
    const int rg = warp % NWR;             // rows rg * RPW .. rg * RPW + RPW - 1
    const int ko = lane / C::LPK;
    const int dq = (lane % C::LPK) * 4;
    const float qscale = rsqrtf((float)D) * 1.4426950408889634f;
    bool ok = true;
    long long x = t_begin;
    for (int si = 0; x < t_end; si++) {
        const int seg = (int)(x / geo.n_t);
        const long long seg_first = (long long)seg * geo.n_t;
        const long long seg_end = std::min<long long>(t_end, seg_first + geo.n_t);
        const int hk = seg % (int)p.n_head_kv;
        const int b = seg / (int)p.n_head_kv;
        const int qb = si & 1;

        int limit[RPW];
#pragma unroll
        for (int k = 0; k < RPW; k++) {
            const int r = rg * RPW + k;
            limit[k] = r < R ? (p.causal ? n_kv - (int)p.n_q + r / G + 1 : n_kv) : 0;
        }
        float m[RPW], l[RPW];
        float4 o[RPW];
#pragma unroll
        for (int k = 0; k < RPW; k++) {
            m[k] = -INFINITY;
            l[k] = 0.f;
            o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (ok && !(ok = mbar_wait(&sm.q_full[qb], (si >> 1) & 1, err))) *(volatile int*)&sm.abort_flag = 1;
        const float(*qs)[D] = &sm.q[qb][rg * RPW];

        if constexpr (KT && RPW == 2) {
            // ---------------------------------------------------------------------------
            // Fast path for the transposed key cache with two query rows per warp (GQA
            // groups of 5-8 rows): lane = (kg, dg) owns keys 4kg..4kg+3 of the tile and the
            // float4 chunks dg, dg + 4, ... of the head dimension. K^T rows are read with
            // 128-bit loads (a quarter-warp reads one contiguous 128-byte row), both rows'
            // partial dots run as packed f32x2 FMAs, and two shuffles add the four
            // quarters. P.V also runs both rows per packed FMA.
            const int kg = lane & 7, dg = lane >> 3;
            float2 o2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                            make_float2(0.f, 0.f)};    // [dim j of this lane's 4][row pair]
            float2 m2 = make_float2(-INFINITY, -INFINITY), l2 = make_float2(0.f, 0.f);
            const long long i0f = x - t_begin;
            const long long firstf = i0f + ((team - (int)(i0f % NT)) + NT) % NT;
            float2* ps = reinterpret_cast<float2*>(&sm.p[warp][0][0]);  // [TK] row pairs
            for (long long i = firstf; ok && t_begin + i < seg_end; i += NT) {
                const int s = (int)(i % C::NS);
                if (!(ok = mbar_wait(&sm.full[s], (uint32_t)(i / C::NS) & 1, err))) {
                    if (lane == 0) *(volatile int*)&sm.abort_flag = 1;
                    break;
                }
                const int t0 = (int)(t_begin + i - seg_first) * TK;
                const float* kt = sm.k[s];
                const float* vt = sm.v[s];
                float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f)};  // [key j][row pair]
#pragma unroll
                for (int mch = 0; mch < D / 16; mch++) {
                    const int c = 4 * mch + dg;
                    const float4 qa = *reinterpret_cast<const float4*>(&qs[0][4 * c]);
                    const float4 qb4 = *reinterpret_cast<const float4*>(&qs[1][4 * c]);
                    const float qa_[4] = {qa.x, qa.y, qa.z, qa.w};
                    const float qb_[4] = {qb4.x, qb4.y, qb4.z, qb4.w};
#pragma unroll
                    for (int ii = 0; ii < 4; ii++) {
                        const float4 kv = *reinterpret_cast<const float4*>(kt + (4 * c + ii) * TK + 4 * kg);
                        const float2 qq = make_float2(qa_[ii], qb_[ii]);
                        acc[0] = __ffma2_rn(qq, make_float2(kv.x, kv.x), acc[0]);
                        acc[1] = __ffma2_rn(qq, make_float2(kv.y, kv.y), acc[1]);
                        acc[2] = __ffma2_rn(qq, make_float2(kv.z, kv.z), acc[2]);
                        acc[3] = __ffma2_rn(qq, make_float2(kv.w, kv.w), acc[3]);
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
#pragma unroll
                    for (int off = 8; off < 32; off <<= 1) {
                        acc[j].x += __shfl_xor_sync(0xffffffffu, acc[j].x, off);
                        acc[j].y += __shfl_xor_sync(0xffffffffu, acc[j].y, off);
                    }
                }
                // online softmax over the tile's 32 keys, both rows
                float xs0[4], xs1[4];
                float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int t = t0 + 4 * kg + j;
                    xs0[j] = (t < n_kv && t < limit[0]) ? acc[j].x * qscale : -INFINITY;
                    xs1[j] = (t < n_kv && t < limit[1]) ? acc[j].y * qscale : -INFINITY;
                    mx0 = fmaxf(mx0, xs0[j]);
                    mx1 = fmaxf(mx1, xs1[j]);
                }
#pragma unroll
                for (int off = 1; off < 8; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                const float mn0 = fmaxf(m2.x, mx0), mn1 = fmaxf(m2.y, mx1);
                const float c0 = (mn0 == -INFINITY) ? 1.f : exp2_approx(m2.x - mn0);
                const float c1 = (mn1 == -INFINITY) ? 1.f : exp2_approx(m2.y - mn1);
                float p0[4], p1[4], s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    p0[j] = mn0 == -INFINITY ? 0.f : exp2_approx(xs0[j] - mn0);
                    p1[j] = mn1 == -INFINITY ? 0.f : exp2_approx(xs1[j] - mn1);
                    s0 += p0[j];
                    s1 += p1[j];
                }
                // the four quarters hold the same keys: only quarter 0 counts them
                l2.x = l2.x * c0 + (dg == 0 ? s0 : 0.f);
                l2.y = l2.y * c1 + (dg == 0 ? s1 : 0.f);
                m2 = make_float2(mn0, mn1);
                const float2 cc = make_float2(c0, c1);
#pragma unroll
                for (int j = 0; j < 4; j++) o2[j] = __fmul2_rn(o2[j], cc);
                if (dg == 0) {
                    float4* dst = reinterpret_cast<float4*>(ps + 4 * kg);
                    dst[0] = make_float4(p0[0], p1[0], p0[1], p1[1]);
                    dst[1] = make_float4(p0[2], p1[2], p0[3], p1[3]);
                }
                __syncwarp();
                // P.V: D/4 lanes per value row, both rows per packed FMA
                const int tt_end = min(TK, n_kv - t0);
#pragma unroll 4
                for (int tt = ko; tt < tt_end; tt += C::KPS) {
                    const float4 vv = *reinterpret_cast<const float4*>(vt + tt * D + dq);
                    const float2 pp2 = ps[tt];
                    o2[0] = __ffma2_rn(pp2, make_float2(vv.x, vv.x), o2[0]);
                    o2[1] = __ffma2_rn(pp2, make_float2(vv.y, vv.y), o2[1]);
                    o2[2] = __ffma2_rn(pp2, make_float2(vv.z, vv.z), o2[2]);
                    o2[3] = __ffma2_rn(pp2, make_float2(vv.w, vv.w), o2[3]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[s]);
            }
            m[0] = m2.x;
            m[1] = m2.y;
            l[0] = l2.x;
            l[1] = l2.y;
            o[0] = make_float4(o2[0].x, o2[1].x, o2[2].x, o2[3].x);
            o[1] = make_float4(o2[0].y, o2[1].y, o2[2].y, o2[3].y);
        } else {
        // this team's tiles of the segment: local indices i with i % NT == team
        const long long i0 = x - t_begin;
        const long long first = i0 + ((team - (int)(i0 % NT)) + NT) % NT;
        for (long long i = first; ok && t_begin + i < seg_end; i += NT) {
            const int s = (int)(i % C::NS);
            if (!(ok = mbar_wait(&sm.full[s], (uint32_t)(i / C::NS) & 1, err))) {
                if (lane == 0) *(volatile int*)&sm.abort_flag = 1;
                break;
            }
            const int t0 = (int)(t_begin + i - seg_first) * TK;
            const float* kt = sm.k[s];
            const float* vt = sm.v[s];
            // ---- scores of this warp's rows, one lane per key
            // four independent partial sums per row keep the FMA chains short
            float4 sa[RPW];
#pragma unroll
            for (int k = 0; k < RPW; k++) sa[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr (KT) {
#pragma unroll 8
                for (int pp = 0; pp < D; pp += 4) {
                    const float k0 = kt[(pp + 0) * TK + lane], k1 = kt[(pp + 1) * TK + lane];
                    const float k2 = kt[(pp + 2) * TK + lane], k3 = kt[(pp + 3) * TK + lane];
#pragma unroll
                    for (int k = 0; k < RPW; k++) {
                        const float4 qv = *reinterpret_cast<const float4*>(&qs[k][pp]);
                        sa[k].x = fmaf(qv.x, k0, sa[k].x);
                        sa[k].y = fmaf(qv.y, k1, sa[k].y);
                        sa[k].z = fmaf(qv.z, k2, sa[k].z);
                        sa[k].w = fmaf(qv.w, k3, sa[k].w);
                    }
                }
            } else {
                const float* krow = kt + lane * D;
#pragma unroll 4
                for (int c = 0; c < D / 4; c++) {
                    const int cc = (c + lane) & (D / 4 - 1);  // rotate: conflict-free rows
                    const float4 kv = *reinterpret_cast<const float4*>(krow + 4 * cc);
#pragma unroll
                    for (int k = 0; k < RPW; k++) {
                        const float4 qv = *reinterpret_cast<const float4*>(&qs[k][4 * cc]);
                        sa[k].x = fmaf(qv.x, kv.x, sa[k].x);
                        sa[k].y = fmaf(qv.y, kv.y, sa[k].y);
                        sa[k].z = fmaf(qv.z, kv.z, sa[k].z);
                        sa[k].w = fmaf(qv.w, kv.w, sa[k].w);
                    }
                }
            }
            float sc[RPW];
#pragma unroll
            for (int k = 0; k < RPW; k++) sc[k] = (sa[k].x + sa[k].y) + (sa[k].z + sa[k].w);
            // ---- online softmax per row (base 2)
            const int t = t0 + lane;
#pragma unroll
            for (int k = 0; k < RPW; k++) {
                const float xv = (t < n_kv && t < limit[k]) ? sc[k] * qscale : -INFINITY;
                const float tmax = warp_max(xv);
                const float m_new = fmaxf(m[k], tmax);
                float pt = 0.f;
                if (m_new != -INFINITY) {
                    const float corr = exp2_approx(m[k] - m_new);
                    pt = exp2_approx(xv - m_new);
                    l[k] = l[k] * corr + pt;
                    o[k].x *= corr;
                    o[k].y *= corr;
                    o[k].z *= corr;
                    o[k].w *= corr;
                    m[k] = m_new;
                }
                sm.p[warp][k][lane] = pt;
            }
            __syncwarp();
            // ---- P.V
            const int tt_end = min(TK, n_kv - t0);
#pragma unroll 4
            for (int tt = ko; tt < tt_end; tt += C::KPS) {
                const float4 vv = *reinterpret_cast<const float4*>(vt + tt * D + dq);
#pragma unroll
                for (int k = 0; k < RPW; k++) {
                    const float pt = sm.p[warp][k][tt];
                    o[k].x = fmaf(pt, vv.x, o[k].x);
                    o[k].y = fmaf(pt, vv.y, o[k].y);
                    o[k].z = fmaf(pt, vv.z, o[k].z);
                    o[k].w = fmaf(pt, vv.w, o[k].w);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[s]);
        }
        }

        // ---- merge the teams' states for this segment (each warp holds its rows)
#pragma unroll
        for (int k = 0; k < RPW; k++) {
            const int r = rg * RPW + k;
#pragma unroll
            for (int off = C::LPK; off < 32; off <<= 1) {
                o[k].x += __shfl_xor_sync(0xffffffffu, o[k].x, off);
                o[k].y += __shfl_xor_sync(0xffffffffu, o[k].y, off);
                o[k].z += __shfl_xor_sync(0xffffffffu, o[k].z, off);
                o[k].w += __shfl_xor_sync(0xffffffffu, o[k].w, off);
            }
            const float lr = warp_sum(l[k]);
            if (lane < C::LPK) *reinterpret_cast<float4*>(&sm.mo[team][r][dq]) = o[k];
            if (lane == 0) {
                sm.mm[team][r] = m[k];
                sm.ml[team][r] = lr;
            }
        }
        named_barrier(1, C::NW * 32);
        if (threadIdx.x == 0) mbar_arrive(&sm.q_empty[qb]);  // q buffer free for the producer
        const int c_first = owner_of(seg_first, geo, gridDim.x);
        const int c_last = owner_of(seg_first + geo.n_t - 1, geo, gridDim.x);
        const int n_pieces = c_last - c_first + 1;
        const int piece = blockIdx.x - c_first;
        float* part_seg = p.ws + (size_t)seg * geo.p_max * R * (D + 2);
        for (int e = threadIdx.x; e < R * D; e += C::NW * 32) {
            const int r = e / D, pp = e % D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NT; w++) M = fmaxf(M, sm.mm[w][r]);
            float L = 0.f, O = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < NT; w++) {
                    const float mw = sm.mm[w][r];
                    const float ew = mw == -INFINITY ? 0.f : exp2_approx(mw - M);
                    L += sm.ml[w][r] * ew;
                    O += sm.mo[w][r][pp] * ew;
                }
            }
            if (n_pieces == 1) {
                p.out[(size_t)b * p.out_bs + (size_t)(r / G) * p.out_stride + (hk * G + (r % G)) * D + pp] =
                    L > 0.f ? O / L : 0.f;
            } else {
                float* part = part_seg + ((size_t)piece * R + r) * (D + 2);
                part[2 + pp] = O;
                if (pp == 0) {
                    part[0] = M;
                    part[1] = L;
                }
            }
        }
        if (n_pieces > 1) {
            // the last CTA to finish this segment merges its pieces: the barrier makes every
            // thread's partial visible to thread 0, whose device-scope fence orders them
            // before its ticket
            named_barrier(1, C::NW * 32);
            if (threadIdx.x == 0) {
                __threadfence();
                const int done = atomicAdd(&counters[seg], 1);
                sm.last = done == n_pieces - 1;
                if (sm.last) counters[seg] = 0;  // ready for the next call
                __threadfence();
            }
            named_barrier(1, C::NW * 32);
            if (sm.last) {
                constexpr int PM = 8;  // pieces merged per pass (loads issued together)
                for (int e = threadIdx.x; e < R * D; e += C::NW * 32) {
                    const int r = e / D, pp = e % D;
                    float M = -INFINITY, L = 0.f, O = 0.f;
                    for (int pc0 = 0; pc0 < n_pieces; pc0 += PM) {
                        float mp[PM], lp[PM], op[PM];
#pragma unroll
                        for (int u = 0; u < PM; u++) {
                            mp[u] = -INFINITY;
                            lp[u] = op[u] = 0.f;
                            if (pc0 + u < n_pieces) {
                                const float* part = part_seg + ((size_t)(pc0 + u) * R + r) * (D + 2);
                                mp[u] = __ldcg(part);
                                lp[u] = __ldcg(part + 1);
                                op[u] = __ldcg(part + 2 + pp);
                            }
                        }
                        float Mn = M;
#pragma unroll
                        for (int u = 0; u < PM; u++) Mn = fmaxf(Mn, mp[u]);
                        if (Mn == -INFINITY) continue;
                        const float cm = M == -INFINITY ? 0.f : exp2_approx(M - Mn);
                        L *= cm;
                        O *= cm;
#pragma unroll
                        for (int u = 0; u < PM; u++) {
                            const float ew = mp[u] == -INFINITY ? 0.f : exp2_approx(mp[u] - Mn);
                            L += lp[u] * ew;
                            O += op[u] * ew;
                        }
                        M = Mn;
                    }
                    p.out[(size_t)b * p.out_bs + (size_t)(r / G) * p.out_stride + (hk * G + (r % G)) * D + pp] =
                        L > 0.f ? O / L : 0.f;
                }
            }
        }
        named_barrier(1, C::NW * 32);  // merge buffers reused by the next segment
        if (*(volatile int*)&sm.abort_flag) break;
        x = seg_end;
    }
}

}  // namespace dec_tma

// ---- host side -------------------------------------------------------------------------------

// f32 3-d map: dims (inner, rows, batch) with the given row and batch strides in elements.
static bool map3(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t batch,
                 uint64_t row_stride, uint64_t batch_stride, uint32_t box_inner, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    if (batch < 1) batch = 1;
    if (batch_stride == 0) batch_stride = row_stride * rows;  // a single item: any valid stride
    cuuint64_t dims[3] = {inner, rows, batch};
    cuuint64_t strides[2] = {row_stride * 4, batch_stride * 4};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool decode_tma_supported(const DecodeParams& p) {
    if (!(p.d == 32 || p.d == 64 || p.d == 128)) return false;
    const size_t rows = p.n_q * (p.n_head / p.n_head_kv);
    if (rows == 0 || rows > 8) return false;
    if (((uintptr_t)p.k | (uintptr_t)p.v | (uintptr_t)p.q) & 15) return false;
    if (p.kv_stride % 4 || p.k_bs % 4 || p.v_bs % 4 || p.q_bs % 4 || p.q_stride % 4 || (p.kt_stride && p.kt_stride % 4))
        return false;
    if (p.n_kv >= (1u << 30)) return false;
    return true;
}

// The schedule: one CTA per SM (fewer when there are fewer tiles). With at least as many
// segments as CTAs each CTA takes whole segments; with at least twice as many SMs as
// segments every segment is cut into min(SMs / segments, kMaxPieces) pieces (at most one
// per tile), one per CTA; otherwise equal ranges over all tiles. p_max bounds the pieces of
// a segment. The cap keeps the last CTA's merge short: it folds the pieces 8 at a time, one
// dependent round of L2 loads per 8, so at one sequence (2 segments of 71 tiles at
// Qwen2.5-1.5B) 16 pieces of ~4 tiles beat 71 pieces of one tile.
constexpr long long kMaxPieces = 16;
static void decode_tma_schedule(size_t n_batch, size_t n_head_kv, size_t n_kv, int sm_count, int* grid, int* p_max,
                                int* mode, int* pieces) {
    const long long n_t = std::max<long long>(1, (long long)((n_kv + dec_tma::TK - 1) / dec_tma::TK));
    const long long segs = std::max<long long>(1, (long long)(n_batch * n_head_kv));
    const long long total = n_t * segs;
    const long long sms = std::max(1, sm_count);
    *pieces = 1;
    if (segs >= sms) {
        *grid = (int)sms;
        *mode = 1;
        *p_max = 1;
    } else if (2 * segs <= sms && n_t >= 2) {
        const long long pc = std::min<long long>(std::min<long long>(sms / segs, n_t), kMaxPieces);
        *grid = (int)(segs * pc);
        *mode = 2;
        *pieces = (int)pc;
        *p_max = (int)pc;
    } else {
        *grid = (int)std::max<long long>(1, std::min<long long>(sms, total));
        *mode = 0;
        *p_max = (int)((*grid + segs - 1) / segs) + 1;
    }
}

void decode_tma_plan(size_t n_batch, size_t n_head_kv, size_t n_kv, int sm_count, int* grid, int* p_max) {
    int mode = 0, pieces = 1;
    decode_tma_schedule(n_batch, n_head_kv, n_kv, sm_count, grid, p_max, &mode, &pieces);
}

size_t decode_tma_workspace_bytes(size_t n_batch, size_t n_head_kv, size_t rows, size_t d, int p_max) {
    const size_t segs = n_batch * n_head_kv;
    const size_t parts = segs * (size_t)p_max * rows * (d + 2) * sizeof(float);
    return ((parts + 255) / 256) * 256 + segs * sizeof(int);
}

template <int D, bool KT>
static int launch_d(const DecodeParams& p, size_t n_batch, int rmax, int grid, int p_max, int mode, int pieces,
                    int* counters, int* err, cudaStream_t st) {
    CUtensorMap mk, mv;
    const uint64_t rows_kv = p.n_kv ? p.n_kv : 1;
    bool okm;
    if (KT)
        okm = map3(&mk, p.k, p.kt_stride, p.n_head_kv * D, n_batch, p.kt_stride, p.k_bs, dec_tma::TK, D);
    else
        okm = map3(&mk, p.k, p.kv_stride, rows_kv, n_batch, p.kv_stride, p.k_bs, D, dec_tma::TK);
    okm = okm && map3(&mv, p.v, p.kv_stride, rows_kv, n_batch, p.kv_stride, p.v_bs, D, dec_tma::TK);
    if (!okm) return -1;
    dec_tma::Geo geo;
    geo.n_t = (int)((p.n_kv + dec_tma::TK - 1) / dec_tma::TK);
    geo.n_segs = (int)(n_batch * p.n_head_kv);
    geo.total = (long long)geo.n_t * geo.n_segs;
    geo.p_max = p_max;
    geo.mode = mode;
    geo.pieces = pieces;
    auto go = [&](auto kern, size_t smem, int threads) -> int {
        // the shared-memory opt-in, once per device and kernel
        static std::mutex mu;
        static std::set<std::pair<int, const void*>> opted;
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return -1;
        {
            std::lock_guard<std::mutex> lk(mu);
            const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kern));
            if (!opted.count(key)) {
                if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                    return -1;
                opted.insert(key);
            }
        }
        if (launch_chained_smem(kern, dim3(grid), dim3(threads), smem, st, mk, mv, p, geo, counters, err) != cudaSuccess)
            return -1;
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    };
    switch (rmax) {
        case 1: return go(dec_tma::decode_tma_kernel<D, KT, 1>, dec_tma::smem_bytes<D, 1>(), dec_tma::Cfg<D, 1>::THREADS);
        case 2: return go(dec_tma::decode_tma_kernel<D, KT, 2>, dec_tma::smem_bytes<D, 2>(), dec_tma::Cfg<D, 2>::THREADS);
        case 4: return go(dec_tma::decode_tma_kernel<D, KT, 4>, dec_tma::smem_bytes<D, 4>(), dec_tma::Cfg<D, 4>::THREADS);
        default: return go(dec_tma::decode_tma_kernel<D, KT, 8>, dec_tma::smem_bytes<D, 8>(), dec_tma::Cfg<D, 8>::THREADS);
    }
}

int decode_tma_launch(const DecodeParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st) {
    if (n_batch == 0 || p.n_q == 0) return 0;
    const size_t rows = p.n_q * (p.n_head / p.n_head_kv);
    const int rmax = rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8;
    int grid = 1, p_max = 1, mode = 0, pieces = 1;
    decode_tma_schedule(n_batch, p.n_head_kv, p.n_kv, sm_count, &grid, &p_max, &mode, &pieces);
    // the segment tickets must start at zero, and the last CTA of each segment puts its
    // ticket back to zero: a kept-zero buffer of the caller's, or the workspace's tail
    // cleared here. Mode 1 (whole segments per CTA) splits no segment and takes no ticket.
    const size_t segs = n_batch * p.n_head_kv;
    const size_t parts = segs * (size_t)p_max * rows * (p.d + 2) * sizeof(float);
    int* counters = p.tickets;
    if (!counters) {
        counters = reinterpret_cast<int*>(reinterpret_cast<char*>(p.ws) + ((parts + 255) / 256) * 256);
        if (mode != 1 && cudaMemsetAsync(counters, 0, segs * sizeof(int), st) != cudaSuccess) return -1;
    }
    const bool kt = p.kt_stride != 0;
    switch (p.d) {
        case 32: return kt ? launch_d<32, true>(p, n_batch, rmax, grid, p_max, mode, pieces, counters, err, st) : launch_d<32, false>(p, n_batch, rmax, grid, p_max, mode, pieces, counters, err, st);
        case 64: return kt ? launch_d<64, true>(p, n_batch, rmax, grid, p_max, mode, pieces, counters, err, st) : launch_d<64, false>(p, n_batch, rmax, grid, p_max, mode, pieces, counters, err, st);
        case 128: return kt ? launch_d<128, true>(p, n_batch, rmax, grid, p_max, mode, pieces, counters, err, st) : launch_d<128, false>(p, n_batch, rmax, grid, p_max, mode, pieces, counters, err, st);
    }
    return -1;
}

}  // namespace zwg
