// f32 attention kernels on the CUDA cores: a tiled flash kernel for any shape the
// reference's attentionEx accepts (src/ops.zig:562-590), and a split-K decode kernel for
// the memory-bound single-token steps (decoder self/cross attention, src/decoder.zig:184
// and :191; Qwen2 decode over the transposed key cache, src/llm.zig:191-202).
//
// Semantics follow the reference exactly: scores are q.k scaled by 1/sqrt(d), the causal
// limit of query row i is n_kv - n_q + i + 1 (src/ops.zig:534), head h reads kv head
// h / (n_head / n_head_kv) (src/ops.zig:521), rows with no visible key produce zeros.
// Softmax is computed online in base 2 (scores pre-multiplied by log2 e), which equals
// the reference's max-subtracted exp up to f32 rounding.
#include "common.cuh"
#include "kernels.h"

#include <math.h>

namespace zwg {

constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------------------------------------
// Tiled flash kernel. TPR threads share one query row, each holding DPT = 32 dims of q and
// of the output accumulator; key/value tiles of TK keys are staged in shared memory and
// reused by all rows of the block.
// ------------------------------------------------------------------------------------------

template <int TPR>
struct FlashCfg {
    static constexpr int DPT = 32;
    static constexpr int DMAX = TPR * DPT;
    static constexpr int THREADS = 256;
    static constexpr int ROWS = THREADS / TPR;
    static constexpr int TK = 32;
};

template <int TPR>
__global__ void __launch_bounds__(256) flash_f32_kernel(FlashParams p) {
    using C = FlashCfg<TPR>;
    extern __shared__ float4 smem_f4[];
    float* Ks = reinterpret_cast<float*>(smem_f4);   // [TK][DMAX]
    float* Vs = Ks + C::TK * C::DMAX;                // [TK][DMAX]

    const int tid = threadIdx.x;
    const int sub = tid % TPR;            // which 32-dim slice of the row
    const int row_in_blk = tid / TPR;
    const size_t b = blockIdx.z;
    const size_t h = blockIdx.y;
    const size_t hk = h / (p.n_head / p.n_head_kv);
    const size_t row0 = (size_t)blockIdx.x * C::ROWS;
    const size_t row = row0 + row_in_blk;
    const bool active = row < p.n_q;
    const int d = (int)p.d;
    const int dbase = sub * C::DPT;
    const int lane = tid & 31;
    const unsigned group_mask = TPR >= 32 ? 0xffffffffu : (((1u << TPR) - 1u) << (lane & ~(TPR - 1)));

    const float* qb = p.q + b * p.q_bs;
    const float* kb = p.k + b * p.k_bs;
    const float* vb = p.v + b * p.v_bs;
    float* ob = p.out + b * p.out_bs;

    const float scale = rsqrtf((float)d) * kLog2e;
    float q[C::DPT], o[C::DPT];
#pragma unroll
    for (int j = 0; j < C::DPT; j++) {
        int dj = dbase + j;
        q[j] = (active && dj < d) ? qb[row * p.q_stride + h * d + dj] : 0.f;
        o[j] = 0.f;
    }
    float m = -INFINITY, l = 0.f;

    // keys this block needs: up to the causal limit of its last row
    size_t last_row = row0 + C::ROWS - 1;
    if (last_row >= p.n_q) last_row = p.n_q ? p.n_q - 1 : 0;
    const size_t kv_end = p.causal ? (p.n_kv - p.n_q + last_row + 1) : p.n_kv;
    const size_t limit = active ? (p.causal ? p.n_kv - p.n_q + row + 1 : p.n_kv) : 0;

    for (size_t t0 = 0; t0 < kv_end; t0 += C::TK) {
        __syncthreads();
        // stage K and V tiles (zero beyond n_kv and beyond d)
        for (int i = tid; i < C::TK * C::DMAX; i += C::THREADS) {
            int tt, pp;
            if (p.kt_stride) {  // keys transposed: coalesce along t
                tt = i % C::TK;
                pp = i / C::TK;
            } else {
                pp = i % C::DMAX;
                tt = i / C::DMAX;
            }
            size_t t = t0 + tt;
            float kval = 0.f, vval = 0.f;
            if (t < p.n_kv && pp < d) {
                kval = p.kt_stride ? kb[(hk * d + pp) * p.kt_stride + t]
                                   : kb[t * p.kv_stride + hk * d + pp];
                vval = vb[t * p.kv_stride + hk * d + pp];
            }
            Ks[tt * C::DMAX + pp] = kval;
            Vs[tt * C::DMAX + pp] = vval;
        }
        __syncthreads();
        // the TPR threads of a row agree on this test, so the shuffles below only ever
        // involve threads that all take the branch
        if (!active || t0 >= limit) continue;
        float s[C::TK];
        float tmax = -INFINITY;
#pragma unroll
        for (int tt = 0; tt < C::TK; tt++) {
            const float4* kr = reinterpret_cast<const float4*>(Ks + tt * C::DMAX + dbase);
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < C::DPT / 4; j++) {
                float4 kv = kr[j];
                acc = fmaf(q[4 * j + 0], kv.x, acc);
                acc = fmaf(q[4 * j + 1], kv.y, acc);
                acc = fmaf(q[4 * j + 2], kv.z, acc);
                acc = fmaf(q[4 * j + 3], kv.w, acc);
            }
#pragma unroll
            for (int off = 1; off < TPR; off <<= 1) acc += __shfl_xor_sync(group_mask, acc, off);
            s[tt] = (t0 + tt < limit) ? acc * scale : -INFINITY;
            tmax = fmaxf(tmax, s[tt]);
        }
        const float m_new = fmaxf(m, tmax);
        const float corr = (m == -INFINITY) ? 0.f : exp2_approx(m - m_new);
        l *= corr;
#pragma unroll
        for (int j = 0; j < C::DPT; j++) o[j] *= corr;
#pragma unroll
        for (int tt = 0; tt < C::TK; tt++) {
            const float pt = exp2_approx(s[tt] - m_new);
            l += pt;
            const float4* vr = reinterpret_cast<const float4*>(Vs + tt * C::DMAX + dbase);
#pragma unroll
            for (int j = 0; j < C::DPT / 4; j++) {
                float4 vv = vr[j];
                o[4 * j + 0] = fmaf(pt, vv.x, o[4 * j + 0]);
                o[4 * j + 1] = fmaf(pt, vv.y, o[4 * j + 1]);
                o[4 * j + 2] = fmaf(pt, vv.z, o[4 * j + 2]);
                o[4 * j + 3] = fmaf(pt, vv.w, o[4 * j + 3]);
            }
        }
        m = m_new;
    }
    if (!active) return;
    const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
    for (int j = 0; j < C::DPT; j++) {
        int dj = dbase + j;
        if (dj < d) ob[row * p.out_stride + h * d + dj] = o[j] * inv;
    }
}

// ------------------------------------------------------------------------------------------
// Split-K decode kernel. One CTA = 4 warps over one (item, kv head, key chunk); all
// R = n_q * group query rows that read this kv head are processed together, so each K/V
// byte is read once per group. Warps take tiles of keys round-robin:
//   KT layout: 128 keys per tile, a lane owns 4 consecutive keys and reads K^T rows with
//              128-bit loads along the position axis;
//   row layout: 32 keys per tile, a lane owns one key row and reads it with 128-bit loads.
// Scores -> online softmax (warp max, lane-partial sums) -> probabilities through shared
// memory -> P.V with D/4 lanes per value row (128-bit loads). The 4 warps merge in shared
// memory; with more than one split, (max, sum, acc) partials go to the workspace and
// decode_combine_kernel merges them.
// ------------------------------------------------------------------------------------------

template <int D, bool KT>
struct DecodeCfg {
    static constexpr int WARPS = 4;
    static constexpr int TILE = KT ? 128 : 32;
    static constexpr int KPL = KT ? 4 : 1;          // keys per lane in the score phase
    static constexpr int LPK = D / 4;               // lanes per value row in the P.V phase
    static constexpr int KPS = 32 / LPK;            // value rows per warp step
};

template <int D, bool KT, int RMAX>
__global__ void __launch_bounds__(128) decode_f32_kernel(DecodeParams p) {
    using C = DecodeCfg<D, KT>;
    __shared__ __align__(16) float q_s[RMAX][D];
    __shared__ __align__(16) float p_s[C::WARPS][RMAX][C::TILE];
    __shared__ float m_s[C::WARPS][RMAX], l_s[C::WARPS][RMAX];
    __shared__ __align__(16) float o_s[C::WARPS][RMAX][D];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int split = blockIdx.x;
    const size_t hk = blockIdx.y;
    const size_t b = blockIdx.z;
    const int G = (int)(p.n_head / p.n_head_kv);
    const int R = (int)p.n_q * G;

    const float* qb = p.q + b * p.q_bs;
    const float* kb = p.k + b * p.k_bs;
    const float* vb = p.v + b * p.v_bs;

    // q rows of this kv head, pre-scaled by log2(e)/sqrt(d); row r = qi * G + g
    const float scale = rsqrtf((float)D) * kLog2e;
    for (int i = threadIdx.x; i < RMAX * D; i += blockDim.x) {
        int r = i / D, pp = i % D;
        float val = 0.f;
        if (r < R) {
            int qi = r / G, g = r % G;
            val = qb[(size_t)qi * p.q_stride + (hk * G + g) * D + pp] * scale;
        }
        q_s[r][pp] = val;
    }
    __syncthreads();

    int limit[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; r++) {
        int qi = r / G;
        limit[r] = r < R ? (p.causal ? (int)(p.n_kv - p.n_q) + qi + 1 : (int)p.n_kv) : 0;
    }

    float m[RMAX], l[RMAX];
    float4 o[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; r++) {
        m[r] = -INFINITY;
        l[r] = 0.f;
        o[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    const int chunk_begin = split * p.chunk;
    int chunk_end = chunk_begin + p.chunk;
    if (chunk_end > (int)p.n_kv) chunk_end = (int)p.n_kv;
    const int ko = lane / C::LPK;
    const int dq = (lane % C::LPK) * 4;

    for (int t0 = chunk_begin + warp * C::TILE; t0 < chunk_end; t0 += C::WARPS * C::TILE) {
        // ---- scores
        float s[RMAX][C::KPL];
#pragma unroll
        for (int r = 0; r < RMAX; r++)
#pragma unroll
            for (int i = 0; i < C::KPL; i++) s[r][i] = 0.f;
        if constexpr (KT) {
            const int tb = t0 + lane * 4;
            if (tb < (int)p.kt_stride) {
                const float* kp = kb + (hk * D) * p.kt_stride + tb;
#pragma unroll 8
                for (int pp = 0; pp < D; pp++) {
                    const float4 kv = __ldg(reinterpret_cast<const float4*>(kp + (size_t)pp * p.kt_stride));
#pragma unroll
                    for (int r = 0; r < RMAX; r++) {
                        const float qv = q_s[r][pp];
                        s[r][0] = fmaf(qv, kv.x, s[r][0]);
                        s[r][1] = fmaf(qv, kv.y, s[r][1]);
                        s[r][2] = fmaf(qv, kv.z, s[r][2]);
                        s[r][3] = fmaf(qv, kv.w, s[r][3]);
                    }
                }
            }
        } else {
            const int t = t0 + lane;
            if (t < chunk_end) {
                const float4* kp = reinterpret_cast<const float4*>(kb + (size_t)t * p.kv_stride + hk * D);
#pragma unroll 4
                for (int j = 0; j < D / 4; j++) {
                    const float4 kv = __ldg(kp + j);
#pragma unroll
                    for (int r = 0; r < RMAX; r++) {
                        const float4 qv = *reinterpret_cast<const float4*>(&q_s[r][4 * j]);
                        s[r][0] = fmaf(qv.x, kv.x, s[r][0]);
                        s[r][0] = fmaf(qv.y, kv.y, s[r][0]);
                        s[r][0] = fmaf(qv.z, kv.z, s[r][0]);
                        s[r][0] = fmaf(qv.w, kv.w, s[r][0]);
                    }
                }
            }
        }
        // ---- online softmax; probabilities to shared memory
#pragma unroll
        for (int r = 0; r < RMAX; r++) {
            float tmax = -INFINITY;
#pragma unroll
            for (int i = 0; i < C::KPL; i++) {
                const int t = t0 + lane * C::KPL + i;
                if (t >= chunk_end || t >= limit[r]) s[r][i] = -INFINITY;
                tmax = fmaxf(tmax, s[r][i]);
            }
            tmax = warp_max(tmax);
            const float m_new = fmaxf(m[r], tmax);
            if (m_new == -INFINITY) {  // nothing visible yet for this row
#pragma unroll
                for (int i = 0; i < C::KPL; i++) p_s[warp][r][lane * C::KPL + i] = 0.f;
                continue;
            }
            const float corr = exp2_approx(m[r] - m_new);
            m[r] = m_new;
            float psum = 0.f;
#pragma unroll
            for (int i = 0; i < C::KPL; i++) {
                const float pt = exp2_approx(s[r][i] - m_new);
                psum += pt;
                p_s[warp][r][lane * C::KPL + i] = pt;
            }
            l[r] = l[r] * corr + psum;
            o[r].x *= corr;
            o[r].y *= corr;
            o[r].z *= corr;
            o[r].w *= corr;
        }
        __syncwarp();
        // ---- P.V
        int tt_end = chunk_end - t0;
        if (tt_end > C::TILE) tt_end = C::TILE;
#pragma unroll 4
        for (int tt = ko; tt < tt_end; tt += C::KPS) {
            const float4 vv = __ldg(reinterpret_cast<const float4*>(vb + (size_t)(t0 + tt) * p.kv_stride + hk * D + dq));
#pragma unroll
            for (int r = 0; r < RMAX; r++) {
                const float pt = p_s[warp][r][tt];
                o[r].x = fmaf(pt, vv.x, o[r].x);
                o[r].y = fmaf(pt, vv.y, o[r].y);
                o[r].z = fmaf(pt, vv.z, o[r].z);
                o[r].w = fmaf(pt, vv.w, o[r].w);
            }
        }
        __syncwarp();
    }

    // ---- reduce inside the warp: P.V partials over the KPS key groups, sums over lanes
#pragma unroll
    for (int r = 0; r < RMAX; r++) {
#pragma unroll
        for (int off = C::LPK; off < 32; off <<= 1) {
            o[r].x += __shfl_xor_sync(0xffffffffu, o[r].x, off);
            o[r].y += __shfl_xor_sync(0xffffffffu, o[r].y, off);
            o[r].z += __shfl_xor_sync(0xffffffffu, o[r].z, off);
            o[r].w += __shfl_xor_sync(0xffffffffu, o[r].w, off);
        }
        l[r] = warp_sum(l[r]);
        if (lane < C::LPK) *reinterpret_cast<float4*>(&o_s[warp][r][dq]) = o[r];
        if (lane == 0) {
            m_s[warp][r] = m[r];
            l_s[warp][r] = l[r];
        }
    }
    __syncthreads();

    // ---- merge the warps; write the output or this split's partial
    for (int i = threadIdx.x; i < R * D; i += blockDim.x) {
        const int r = i / D, pp = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < C::WARPS; w++) M = fmaxf(M, m_s[w][r]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < C::WARPS; w++) {
                const float e = m_s[w][r] == -INFINITY ? 0.f : exp2_approx(m_s[w][r] - M);
                L += l_s[w][r] * e;
                O += o_s[w][r][pp] * e;
            }
        }
        if (p.n_splits == 1) {
            const int qi = r / G, g = r % G;
            p.out[b * p.out_bs + (size_t)qi * p.out_stride + (hk * G + g) * D + pp] = L > 0.f ? O / L : 0.f;
        } else {
            float* part = p.ws + ((((size_t)b * p.n_head_kv + hk) * p.n_splits + split) * R + r) * (D + 2);
            part[2 + pp] = O;
            if (pp == 0) {
                part[0] = M;
                part[1] = L;
            }
        }
    }
}

// Merge split partials: one block of D threads per (item, kv head, row).
template <int D>
__global__ void decode_combine_kernel(DecodeParams p) {
    const int G = (int)(p.n_head / p.n_head_kv);
    const int R = (int)p.n_q * G;
    const size_t idx = blockIdx.x;
    const int r = (int)(idx % R);
    const size_t hk = (idx / R) % p.n_head_kv;
    const size_t b = idx / R / p.n_head_kv;
    const int pp = threadIdx.x;
    const float* base = p.ws + (((size_t)b * p.n_head_kv + hk) * p.n_splits * R + r) * (D + 2);
    const size_t split_stride = (size_t)R * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < p.n_splits; s++) M = fmaxf(M, base[s * split_stride]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
        for (int s = 0; s < p.n_splits; s++) {
            const float* part = base + s * split_stride;
            const float ms = part[0];
            const float e = ms == -INFINITY ? 0.f : exp2_approx(ms - M);
            L += part[1] * e;
            O += part[2 + pp] * e;
        }
    }
    const int qi = r / G, g = r % G;
    p.out[b * p.out_bs + (size_t)qi * p.out_stride + (hk * G + g) * D + pp] = L > 0.f ? O / L : 0.f;
}

// ------------------------------------------------------------------------------------------
// Host-side launchers
// ------------------------------------------------------------------------------------------

int flash_f32_launch(const FlashParams& p, size_t n_batch, cudaStream_t st) {
    if (p.n_q == 0 || n_batch == 0) return 0;
    auto go = [&](auto kern, int tpr) -> int {
        const int rows = 256 / tpr;
        const size_t smem = 2 * 32 * (size_t)tpr * 32 * sizeof(float);
        if (smem > 48 * 1024)
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -1;
        dim3 grid((unsigned)((p.n_q + rows - 1) / rows), (unsigned)p.n_head, (unsigned)n_batch);
        kern<<<grid, 256, smem, st>>>(p);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    };
    if (p.d <= 32) return go(flash_f32_kernel<1>, 1);
    if (p.d <= 64) return go(flash_f32_kernel<2>, 2);
    if (p.d <= 128) return go(flash_f32_kernel<4>, 4);
    if (p.d <= 256) return go(flash_f32_kernel<8>, 8);
    return -1;
}

bool decode_supported(size_t d, size_t rows, size_t kt_stride) {
    if (!(d == 32 || d == 64 || d == 128)) return false;
    if (rows == 0 || rows > 8) return false;
    if (kt_stride % 4) return false;
    return true;
}

int decode_rmax(size_t rows) {
    return rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8;
}

int decode_combine_launch(const DecodeParams& p, size_t n_batch, cudaStream_t st);

template <int D, bool KT>
static int decode_launch_d(const DecodeParams& p, size_t n_batch, int rmax, cudaStream_t st) {
    dim3 grid((unsigned)p.n_splits, (unsigned)p.n_head_kv, (unsigned)n_batch);
    switch (rmax) {
        case 1: decode_f32_kernel<D, KT, 1><<<grid, 128, 0, st>>>(p); break;
        case 2: decode_f32_kernel<D, KT, 2><<<grid, 128, 0, st>>>(p); break;
        case 4: decode_f32_kernel<D, KT, 4><<<grid, 128, 0, st>>>(p); break;
        default: decode_f32_kernel<D, KT, 8><<<grid, 128, 0, st>>>(p); break;
    }
    if (cudaPeekAtLastError() != cudaSuccess) return -1;
    if (p.n_splits > 1) return decode_combine_launch(p, n_batch, st);
    return 0;
}

int decode_combine_launch(const DecodeParams& p, size_t n_batch, cudaStream_t st) {
    const size_t rows = p.n_q * (p.n_head / p.n_head_kv);
    const unsigned blocks = (unsigned)(n_batch * p.n_head_kv * rows);
    switch (p.d) {
        case 32: decode_combine_kernel<32><<<blocks, 32, 0, st>>>(p); break;
        case 64: decode_combine_kernel<64><<<blocks, 64, 0, st>>>(p); break;
        case 128: decode_combine_kernel<128><<<blocks, 128, 0, st>>>(p); break;
        default: return -1;
    }
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int decode_f32_launch(const DecodeParams& p, size_t n_batch, cudaStream_t st) {
    if (n_batch == 0 || p.n_q == 0) return 0;
    const int rmax = decode_rmax(p.n_q * (p.n_head / p.n_head_kv));
    const bool kt = p.kt_stride != 0;
    switch (p.d) {
        case 32: return kt ? decode_launch_d<32, true>(p, n_batch, rmax, st) : decode_launch_d<32, false>(p, n_batch, rmax, st);
        case 64: return kt ? decode_launch_d<64, true>(p, n_batch, rmax, st) : decode_launch_d<64, false>(p, n_batch, rmax, st);
        case 128: return kt ? decode_launch_d<128, true>(p, n_batch, rmax, st) : decode_launch_d<128, false>(p, n_batch, rmax, st);
    }
    return -1;
}

// Split count: enough CTAs for about four waves of 148 SMs, each CTA at least one tile
// per warp, chunks a multiple of the tile so warps stay aligned with the KT 128-bit loads.
void decode_plan(size_t n_batch, size_t n_head_kv, size_t n_kv, bool kt, int sm_count,
                 int* n_splits, int* chunk) {
    const int tile = kt ? 128 : 32;
    const int min_chunk = tile * 4;
    const size_t items = n_batch * n_head_kv;
    const size_t target = (size_t)sm_count * 8;
    int splits = (int)((target + items - 1) / (items ? items : 1));
    const int max_splits = (int)((n_kv + min_chunk - 1) / min_chunk);
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    int ch = (int)((n_kv + splits - 1) / splits);
    ch = (ch + tile - 1) / tile * tile;
    if (ch < tile) ch = tile;
    splits = (int)((n_kv + ch - 1) / ch);
    if (splits < 1) splits = 1;
    *n_splits = splits;
    *chunk = ch;
}

size_t decode_workspace_floats(size_t n_batch, size_t n_head_kv, size_t rows, int n_splits, size_t d) {
    if (n_splits <= 1) return 0;
    return n_batch * n_head_kv * (size_t)n_splits * rows * (d + 2);
}

}  // namespace zwg
