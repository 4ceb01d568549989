// Split-K decode attention fed by TMA (sm_100a): the memory-bound single-token steps of
// the decoder (self- and cross-attention, src/decoder.zig:184 and :191) and of Qwen2 over
// its transposed key cache (src/llm.zig:191-202).
//
// Work: units of (item, kv head, chunk of keys); a persistent grid deals units to CTAs.
// Every unit covers CH tiles of 32 keys; all R = n_q * group query rows that read the kv
// head are processed together, so each K/V byte is read once per GQA group.
//   warp NW     producer: one thread streams K and V tiles of 32 keys into an NS-slot ring
//               with 2-D/3-D TMA tile loads (no multicast): K^T boxes [d][32] for the
//               transposed cache, row boxes [32][d] otherwise; V boxes [32][d]. Tens of KB
//               in flight per SM with no register cost, which is what an HBM-bound kernel
//               needs.
//   warps 0..NW-1  compute, warp w owns ring slot w (NW = NS): scores with one lane per
//               key, online softmax in base 2 per warp (warp max, lane-partial sums),
//               probabilities through shared memory, P.V with D/4 lanes per value row.
//               At the end of a unit the warps merge their (max, sum, accumulator) states in
//               shared memory; a unit that spans the whole key range writes the output, the
//               others write a partial that decode_combine_kernel merges.
// Keys past n_kv (zero fill or finite cache junk) are masked to -inf per row, with the
// causal limit n_kv - n_q + i + 1 of query row i (src/ops.zig:534).
//
// Every mbarrier wait is bounded (sm100::mbar_wait); a timeout records kErrTimeout in the
// error word and the CTA skips to its exit.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace zwg {

using namespace sm100;

namespace dec_tma {

constexpr int TK = 32;  // keys per tile

template <int D>
struct Cfg {
    static constexpr int NS = D >= 128 ? 5 : 8;              // ring slots = compute warps
    static constexpr int NW = NS;
    static constexpr int THREADS = (NW + 1) * 32;
    static constexpr uint32_t K_BYTES = TK * D * 4;
    static constexpr uint32_t V_BYTES = TK * D * 4;
    static constexpr int LPK = D / 4;                         // lanes per value row (P.V)
    static constexpr int KPS = 32 / LPK;                      // value rows per warp step
};

template <int D, int RMAX>
struct Smem {
    float k[Cfg<D>::NS][TK * D];      // K^T: [D][32]; rows: [32][D]
    float v[Cfg<D>::NS][TK * D];      // [32][D]
    float q[RMAX][D];                 // pre-scaled by log2(e)/sqrt(d)
    float p[Cfg<D>::NW][RMAX][TK];
    float mo[Cfg<D>::NW][RMAX][D];    // merge: accumulators
    float mm[Cfg<D>::NW][RMAX];       // merge: maxima
    float ml[Cfg<D>::NW][RMAX];       // merge: sums
    uint64_t full[Cfg<D>::NS], empty[Cfg<D>::NS];
    int abort_flag;
};

template <int D, int RMAX>
constexpr size_t smem_bytes() {
    return sizeof(Smem<D, RMAX>) + 128;
}

struct Geo {
    int n_units, n_chunks, ch_tiles;
};

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int D, bool KT, int RMAX>
__global__ void __launch_bounds__(Cfg<D>::THREADS, 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      DecodeParams p, Geo geo, int* err) {
    using C = Cfg<D>;
    extern __shared__ uint8_t smem_raw[];
    Smem<D, RMAX>& sm = *reinterpret_cast<Smem<D, RMAX>*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = (int)(p.n_head / p.n_head_kv);
    const int R = (int)p.n_q * G;
    const int n_kv = (int)p.n_kv;
    const int chunk_keys = geo.ch_tiles * TK;

    if (threadIdx.x == 0) sm.abort_flag = err ? *(volatile int*)err : 0;
    __syncthreads();
    if (sm.abort_flag) return;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NS; s++) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == C::NW) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tmap(&tm_k);
            prefetch_tmap(&tm_v);
            uint32_t g = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < geo.n_units; u += gridDim.x) {
                const int chunk = u % geo.n_chunks;
                const int hk = (u / geo.n_chunks) % (int)p.n_head_kv;
                const int b = u / geo.n_chunks / (int)p.n_head_kv;
                const int t_begin = chunk * chunk_keys;
                const int t_end = min(n_kv, t_begin + chunk_keys);
                for (int t0 = t_begin; t0 < t_end; t0 += TK, g++) {
                    const int s = g % C::NS;
                    if (g >= (uint32_t)C::NS && !(ok = mbar_wait(&sm.empty[s], ((g / C::NS) - 1) & 1, err))) break;
                    mbar_arrive_expect_tx(&sm.full[s], C::K_BYTES + C::V_BYTES);
                    if (KT) tma_load_3d(&tm_k, &sm.full[s], sm.k[s], t0, hk * D, b);
                    else tma_load_3d(&tm_k, &sm.full[s], sm.k[s], hk * D, t0, b);
                    tma_load_3d(&tm_v, &sm.full[s], sm.v[s], hk * D, t0, b);
                }
            }
        }
        return;
    }

    // -------------------------------------------------------------------- compute warps
    const int ko = lane / C::LPK;
    const int dq = (lane % C::LPK) * 4;
    const float qscale = rsqrtf((float)D) * 1.4426950408889634f;
    uint32_t g = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < geo.n_units; u += gridDim.x) {
        const int chunk = u % geo.n_chunks;
        const int hk = (u / geo.n_chunks) % (int)p.n_head_kv;
        const int b = u / geo.n_chunks / (int)p.n_head_kv;
        const int t_begin = chunk * chunk_keys;
        const int t_end = min(n_kv, t_begin + chunk_keys);
        const int n_t = (t_end - t_begin + TK - 1) / TK;

        // q rows of this kv head, row r = qi * G + g
        const float* qb = p.q + (size_t)b * p.q_bs;
        for (int i = threadIdx.x; i < RMAX * D; i += C::NW * 32) {
            const int r = i / D, pp = i % D;
            float val = 0.f;
            if (r < R) val = qb[(size_t)(r / G) * p.q_stride + (hk * G + (r % G)) * D + pp] * qscale;
            sm.q[r][pp] = val;
        }
        named_barrier(1, C::NW * 32);

        int limit[RMAX];
#pragma unroll
        for (int r = 0; r < RMAX; r++)
            limit[r] = r < R ? (p.causal ? n_kv - (int)p.n_q + r / G + 1 : n_kv) : 0;
        float m[RMAX], l[RMAX];
        float4 o[RMAX];
#pragma unroll
        for (int r = 0; r < RMAX; r++) {
            m[r] = -INFINITY;
            l[r] = 0.f;
            o[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        }

        // tiles of this unit are global tiles g .. g + n_t - 1; this warp owns slot `warp`
        for (int i = 0; ok && i < n_t; i++) {
            const uint32_t gi = g + i;
            if ((int)(gi % C::NS) != warp) continue;
            if (!(ok = mbar_wait(&sm.full[warp], (gi / C::NS) & 1, err))) {
                if (lane == 0) *(volatile int*)&sm.abort_flag = 1;
                break;
            }
            const int t0 = t_begin + i * TK;
            const float* kt = sm.k[warp];
            const float* vt = sm.v[warp];
            // ---- scores, one lane per key
            float s[RMAX];
#pragma unroll
            for (int r = 0; r < RMAX; r++) s[r] = 0.f;
            if constexpr (KT) {
#pragma unroll 8
                for (int pp = 0; pp < D; pp += 4) {
                    const float k0 = kt[(pp + 0) * TK + lane], k1 = kt[(pp + 1) * TK + lane];
                    const float k2 = kt[(pp + 2) * TK + lane], k3 = kt[(pp + 3) * TK + lane];
#pragma unroll
                    for (int r = 0; r < RMAX; r++) {
                        const float4 qv = *reinterpret_cast<const float4*>(&sm.q[r][pp]);
                        s[r] = fmaf(qv.x, k0, fmaf(qv.y, k1, fmaf(qv.z, k2, fmaf(qv.w, k3, s[r]))));
                    }
                }
            } else {
                const float* krow = kt + lane * D;
#pragma unroll 4
                for (int c = 0; c < D / 4; c++) {
                    const int cc = (c + lane) & (D / 4 - 1);  // rotate: conflict-free rows
                    const float4 kv = *reinterpret_cast<const float4*>(krow + 4 * cc);
#pragma unroll
                    for (int r = 0; r < RMAX; r++) {
                        const float4 qv = *reinterpret_cast<const float4*>(&sm.q[r][4 * cc]);
                        s[r] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, s[r]))));
                    }
                }
            }
            // ---- online softmax per row
            const int t = t0 + lane;
#pragma unroll
            for (int r = 0; r < RMAX; r++) {
                const float x = (t < t_end && t < limit[r]) ? s[r] : -INFINITY;
                const float tmax = warp_max(x);
                const float m_new = fmaxf(m[r], tmax);
                float pt = 0.f;
                if (m_new != -INFINITY) {
                    const float corr = exp2_approx(m[r] - m_new);
                    pt = exp2_approx(x - m_new);
                    l[r] = l[r] * corr + pt;
                    o[r].x *= corr;
                    o[r].y *= corr;
                    o[r].z *= corr;
                    o[r].w *= corr;
                    m[r] = m_new;
                }
                sm.p[warp][r][lane] = pt;
            }
            __syncwarp();
            // ---- P.V
            const int tt_end = min(TK, t_end - t0);
#pragma unroll 4
            for (int tt = ko; tt < tt_end; tt += C::KPS) {
                const float4 vv = *reinterpret_cast<const float4*>(vt + tt * D + dq);
#pragma unroll
                for (int r = 0; r < RMAX; r++) {
                    const float pt = sm.p[warp][r][tt];
                    o[r].x = fmaf(pt, vv.x, o[r].x);
                    o[r].y = fmaf(pt, vv.y, o[r].y);
                    o[r].z = fmaf(pt, vv.z, o[r].z);
                    o[r].w = fmaf(pt, vv.w, o[r].w);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[warp]);
        }
        g += n_t;

        // ---- merge the warps' states
#pragma unroll
        for (int r = 0; r < RMAX; r++) {
#pragma unroll
            for (int off = C::LPK; off < 32; off <<= 1) {
                o[r].x += __shfl_xor_sync(0xffffffffu, o[r].x, off);
                o[r].y += __shfl_xor_sync(0xffffffffu, o[r].y, off);
                o[r].z += __shfl_xor_sync(0xffffffffu, o[r].z, off);
                o[r].w += __shfl_xor_sync(0xffffffffu, o[r].w, off);
            }
            const float lr = warp_sum(l[r]);
            if (lane < C::LPK) *reinterpret_cast<float4*>(&sm.mo[warp][r][dq]) = o[r];
            if (lane == 0) {
                sm.mm[warp][r] = m[r];
                sm.ml[warp][r] = lr;
            }
        }
        named_barrier(1, C::NW * 32);
        const bool whole = geo.n_chunks == 1;
        for (int i = threadIdx.x; i < R * D; i += C::NW * 32) {
            const int r = i / D, pp = i % D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < C::NW; w++) M = fmaxf(M, sm.mm[w][r]);
            float L = 0.f, O = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < C::NW; w++) {
                    const float mw = sm.mm[w][r];
                    const float e = mw == -INFINITY ? 0.f : exp2_approx(mw - M);
                    L += sm.ml[w][r] * e;
                    O += sm.mo[w][r][pp] * e;
                }
            }
            if (whole) {
                p.out[(size_t)b * p.out_bs + (size_t)(r / G) * p.out_stride + (hk * G + (r % G)) * D + pp] =
                    L > 0.f ? O / L : 0.f;
            } else {
                float* part = p.ws + ((((size_t)b * p.n_head_kv + hk) * geo.n_chunks + chunk) * R + r) * (D + 2);
                part[2 + pp] = O;
                if (pp == 0) {
                    part[0] = M;
                    part[1] = L;
                }
            }
        }
        named_barrier(1, C::NW * 32);  // merge buffers and q reused by the next unit
        if (*(volatile int*)&sm.abort_flag) break;  // every compute warp leaves together
    }
}

}  // namespace dec_tma

// ---- host side -------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn() {
    static EncodeTiledFn2 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn2)ptr;
    });
    return fn;
}

// f32 3-d map: dims (inner, rows, batch) with the given row and batch strides in elements.
static bool map3(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t batch,
                 uint64_t row_stride, uint64_t batch_stride, uint32_t box_inner, uint32_t box_rows) {
    EncodeTiledFn2 fn = encode_fn();
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
    if (((uintptr_t)p.k | (uintptr_t)p.v) & 15) return false;
    if (p.kv_stride % 4 || p.k_bs % 4 || p.v_bs % 4 || (p.kt_stride && p.kt_stride % 4)) return false;
    if (p.n_kv >= (1u << 30)) return false;
    return true;
}

void decode_tma_plan(size_t n_batch, size_t n_head_kv, size_t n_kv, int sm_count, int* n_chunks, int* ch_tiles) {
    const size_t segs = n_batch * n_head_kv;
    const int tiles = (int)((n_kv + dec_tma::TK - 1) / dec_tma::TK);
    // about four units per SM, a unit at least 8 tiles (its warps merge once per unit)
    size_t want = (size_t)sm_count * 4;
    int chunks = (int)std::max<size_t>(1, (want + segs - 1) / std::max<size_t>(segs, 1));
    chunks = std::min(chunks, std::max(1, tiles / 8));
    int ch = (tiles + chunks - 1) / chunks;
    if (ch < 1) ch = 1;
    chunks = (tiles + ch - 1) / ch;
    if (chunks < 1) chunks = 1;
    *n_chunks = chunks;
    *ch_tiles = ch;
}

template <int D, bool KT>
static int launch_d(const DecodeParams& p, size_t n_batch, int rmax, int sm_count, int* err, cudaStream_t st) {
    using C = dec_tma::Cfg<D>;
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
    geo.n_chunks = p.n_splits;
    geo.ch_tiles = p.chunk / dec_tma::TK;
    geo.n_units = (int)(n_batch * p.n_head_kv * (size_t)p.n_splits);
    const int grid = std::min(geo.n_units, sm_count);
    auto go = [&](auto kern, size_t smem) -> int {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return -1;
        kern<<<grid, C::THREADS, smem, st>>>(mk, mv, p, geo, err);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    };
    int rc;
    switch (rmax) {
        case 1: rc = go(dec_tma::decode_tma_kernel<D, KT, 1>, dec_tma::smem_bytes<D, 1>()); break;
        case 2: rc = go(dec_tma::decode_tma_kernel<D, KT, 2>, dec_tma::smem_bytes<D, 2>()); break;
        case 4: rc = go(dec_tma::decode_tma_kernel<D, KT, 4>, dec_tma::smem_bytes<D, 4>()); break;
        default: rc = go(dec_tma::decode_tma_kernel<D, KT, 8>, dec_tma::smem_bytes<D, 8>()); break;
    }
    if (rc) return rc;
    if (p.n_splits > 1) return decode_combine_launch(p, n_batch, st);
    return 0;
}

int decode_tma_launch(const DecodeParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st) {
    if (n_batch == 0 || p.n_q == 0) return 0;
    const size_t rows = p.n_q * (p.n_head / p.n_head_kv);
    const int rmax = rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8;
    const bool kt = p.kt_stride != 0;
    switch (p.d) {
        case 32: return kt ? launch_d<32, true>(p, n_batch, rmax, sm_count, err, st) : launch_d<32, false>(p, n_batch, rmax, sm_count, err, st);
        case 64: return kt ? launch_d<64, true>(p, n_batch, rmax, sm_count, err, st) : launch_d<64, false>(p, n_batch, rmax, sm_count, err, st);
        case 128: return kt ? launch_d<128, true>(p, n_batch, rmax, sm_count, err, st) : launch_d<128, false>(p, n_batch, rmax, sm_count, err, st);
    }
    return -1;
}

}  // namespace zwg
