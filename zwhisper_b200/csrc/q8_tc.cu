// Q8 products for 16 or more rows of activations on the 5th-generation tensor cores
// (sm_100a): ops.linear with Q8 weights (src/ops.zig:280-306 -> gemm.ntBlockQ,
// src/gemm.zig:268-351) for a decoder step over many windows, an LLM step over many
// sequences, prompt chunks and setAudio's 1500 rows, with the epilogues of
// q8_linear_kernel (store + bias, add into out, tanh GELU), the SiLU pair (gate and up,
// src/llm.zig:206-208), the Qwen2 q/k/v pair (bias, RoPE, q out, K^T scatter and V copy,
// src/llm.zig:179-190, 221-238) and the Whisper decoder's q/k/v product (bias, q out, k and
// v appended to the caches, src/decoder.zig:389-395).
//
//   out[r][j] = epilogue( sum over blocks b of  s[j][b] * sum_{i < 32} x[r][32b + i] * q[j][32b + i] )
//
// The reference's arithmetic is kept: each 32-wide block's dot is formed first and then
// multiplied by the block's scale, as gemm.ntBlockQ does. The tensor cores form the block
// dots from exact products: the int8 weights are exact in bf16, and each f32 activation is
// split into three bf16 pieces whose sum is the activation exactly (its top 8 significant
// bits, the next 8, the last 8: truncations, so each remainder is exact). A block's dot is
// six MMAs (kind::f16, bf16 x bf16, f32 accumulation) into one TMEM accumulator: its two
// K16 slices against each piece, the weights reused as A. Every product is exact; only the
// f32 sums round, in another order than the reference's (the same bound as the CUDA-core
// kernels: a few f32 ulps of the sum of |terms|).
//
// Tile: 128 weight rows (TMEM lanes) x 128 activation rows (more than 64 rows of x) or x 64
// activation rows with the three pieces stacked along N instead of K (16-64 rows: one N192
// MMA per K16 slice into a 192-column accumulator whose three 64-column parts the scalers
// sum; a third of the MMAs of the 128-row form, most of whose rows would be past m). A CTA
// walks its k range in steps of 64 (two Q8 blocks). The 128-row form:
//   warp 0      TMA producer: int8 weights [128 rows][64] (two [64][64] boxes for the SiLU
//               pair: gate rows, then up rows) and f32 activations [128 rows][64] into a
//               2-stage raw ring; rows past n or m are zero-filled.
//   warp 1      allocates 512 TMEM columns (four 128-column block accumulators); lane 0
//               issues the six MMAs of each Q8 block.
//   warps 2-9   convert a raw stage into the MMA operands (2-stage ring, 128-byte swizzle):
//               int8 -> bf16 exactly (through f32 2^23 + u - (2^23 + 128)), f32 -> three
//               bf16 pieces; activation rows past m are zero after a stage's first use and
//               are not converted again.
//   warps 10-17 one weight row (TMEM lane) and 64 of the 128 activation rows per thread: per
//               block, the accumulator times the block's scale added into 64 f32 registers;
//               then the epilogue.
// Split-K: when the tiles alone would leave SMs idle, a cluster of ks CTAs (1 x 1 x ks)
// takes one tile, each CTA a contiguous range of k steps; the partial tiles are reduced in
// rank order through distributed shared memory (deterministic, no workspace).
// Every mbarrier wait is bounded; after a timeout the CTA drains its own copies and MMAs
// (bounded), every thread still reaches the cluster barriers, and TMEM is freed.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "api_internal.h"
#include "chain.cuh"
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace zwg {
namespace q8tc {

using namespace sm100;

constexpr int BM = 128;          // weight rows per tile (TMEM lanes)
constexpr int BK = 64;           // k per step: two Q8 blocks
constexpr int NP = 3;            // bf16 pieces of an activation
constexpr int MAX_KS = 8;        // CTAs per cluster (k splits)
constexpr int CONV_WARPS = 8;
constexpr int SCALE_WARPS = 8;
constexpr int THREADS = 32 * (2 + CONV_WARPS + SCALE_WARPS);
constexpr int CONV_THREADS = 32 * CONV_WARPS;
constexpr int SCALE_THREADS = 32 * SCALE_WARPS;
constexpr int SCALE_WARP0 = 2 + CONV_WARPS;
constexpr uint32_t RAW_W = BM * BK;               // int8
constexpr uint32_t CV_A = BM * BK * 2;            // bf16, 128-byte rows
constexpr uint32_t TMEM_COLS = 512;
constexpr int PART_LD = BM + 4;                   // row stride of the split-K partial tile (floats)
constexpr int PAIR_LD = BM / 2 + 4;               // row stride of the SiLU pair's exchange (floats)

// The two tile forms. Large (more than 64 rows of x): 128 activation rows, the pieces along
// K, one 128-column accumulator per Q8 block (six N128 MMAs per block). Small (16-64 rows):
// 64 activation rows, the pieces stacked along N (rows p * 64 + r of the B operand), one
// 192-column accumulator per block holding the three pieces' dots side by side, summed by
// the scalers (two N192 MMAs per block: a third of the large form's MMAs, where those
// would mostly multiply rows past m).
template <bool SMALL>
struct Tr {
    static constexpr int TN = SMALL ? 64 : 128;            // activation rows per tile
    static constexpr int NSR = SMALL ? 3 : 2;              // raw stages
    static constexpr int NSC = SMALL ? 3 : 2;              // converted stages
    static constexpr int NSLOT = SMALL ? 2 : 4;            // block accumulators in TMEM
    static constexpr uint32_t ACC = SMALL ? NP * 64 : 128; // TMEM columns of one
    static constexpr int COLS = TN / 2;                    // activation rows per scaler thread
    static constexpr uint32_t RAW_X = TN * BK * 4;         // f32
    static constexpr uint32_t CV_P = TN * BK * 2;          // one piece: bf16, 128-byte rows
    static_assert(NSLOT * ACC <= TMEM_COLS, "TMEM columns");
};

template <bool SMALL>
struct Smem {
    using T = Tr<SMALL>;
    uint8_t cv_a[T::NSC][CV_A];
    uint8_t cv_b[T::NSC][NP * T::CV_P];
    uint8_t raw_x[T::NSR][T::RAW_X];
    uint8_t raw_w[T::NSR][RAW_W];
    uint64_t raw_full[T::NSR], raw_empty[T::NSR], cv_full[T::NSC], cv_empty[T::NSC];
    uint64_t acc_full[T::NSLOT], acc_empty[T::NSLOT];
    uint32_t tmem_base;
};
template <bool SMALL>
constexpr size_t smem_bytes() { return sizeof(Smem<SMALL>) + 1024; }
static_assert(smem_bytes<false>() <= 227 * 1024 && smem_bytes<true>() <= 227 * 1024, "shared memory of one CTA");
static_assert(Tr<false>::TN * PART_LD * 4 <= Tr<false>::NSC * NP * Tr<false>::CV_P &&
                  Tr<true>::TN * PART_LD * 4 <= Tr<true>::NSC * NP * Tr<true>::CV_P,
              "the split-K partial tile fits in the operand ring");
static_assert(THREADS * 96 <= 65536, "registers");

// Epilogue modes: a plain product, the SiLU pair, and two forms over the three q/k/v
// matrices (a CTA's 128-row tile lies in one of them: tiles of matrix 0, then 1, then 2):
// the Qwen2 RoPE pair (bias, rotation of rows i and i + d/2 of a head, q out, K^T scatter,
// V copy) and the Whisper decoder's q/k/v (bias, q out, k and v appended to the caches).
enum { EPI_PLAIN = 0, EPI_SILU = 1, EPI_ROPE = 2, EPI_QKV = 3 };

struct Args {
    int m, n, k, ks;             // ks: CTAs per cluster
    int mode;                    // LIN_STORE / LIN_ADD / LIN_GELU
    const float* ws;             // scales [n][k/32] (the gate's for the pair)
    const float* wsu;            // the up matrix's scales (pair), else null
    const float* bias;
    const float* bias_u;
    float* out;
    int* err;
    int tiles[3];                // ROPE / QKV: 128-row tiles of each matrix
    PairParams pp;               // ROPE / QKV: the matrices' scales and biases, caches, tables
};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // a in the low half (the lower k)
    return *reinterpret_cast<uint32_t*>(&h);
}

// four int8 (one word) -> two bf16 pairs, exactly: byte u = q + 128 placed under the
// exponent of 2^23 gives 2^23 + u, minus (2^23 + 128) is q
__device__ __forceinline__ void int8x4_to_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const float2 nbase = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    // byte i of u as the low mantissa byte of 0x4B0000uu (selectors: byte i, two zero
    // bytes and the exponent byte 0x4B of the second operand)
    const float2 a = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541))), nbase);
    const float2 b = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543))), nbase);
    lo = pack_bf16(a.x, a.y);
    hi = pack_bf16(b.x, b.y);
}

// -(the value truncated to bf16): the top 16 bits, sign flipped
__device__ __forceinline__ float neg_trunc(float v) { return __uint_as_float((__float_as_uint(v) & 0xffff0000u) ^ 0x80000000u); }

// two f32 -> their bf16 pieces (hi, mid, lo pairs; lower k in the low half). Each piece is
// the previous remainder truncated to bf16; remainders are exact in f32 and the last one
// has at most 8 significant bits, so hi + mid + lo == the value exactly.
__device__ __forceinline__ void split3(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
    hi = __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x7632);
    const float2 r1 = __fadd2_rn(make_float2(a, b), make_float2(neg_trunc(a), neg_trunc(b)));
    mid = __byte_perm(__float_as_uint(r1.x), __float_as_uint(r1.y), 0x7632);
    const float2 r2 = __fadd2_rn(r1, make_float2(neg_trunc(r1.x), neg_trunc(r1.y)));
    lo = __byte_perm(__float_as_uint(r2.x), __float_as_uint(r2.y), 0x7632);
}

__device__ __forceinline__ float gelu_tanh(float x) {
    const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(u)));
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// the epilogue of one output of a plain product (q8_linear_kernel's)
__device__ __forceinline__ void finish(const Args& a, int row, int col, float v) {
    if (a.bias) v = __fadd_rn(v, __ldg(a.bias + col));
    float* o = a.out + (size_t)row * a.n + col;
    if (a.mode == LIN_ADD) v = __fadd_rn(__ldcg(o), v);
    else if (a.mode == LIN_GELU) v = gelu_tanh(v);
    *o = v;
}

__device__ __forceinline__ void finish_pair(const Args& a, int row, int col, float g, float u) {
    if (a.bias) g = __fadd_rn(g, __ldg(a.bias + col));
    if (a.bias_u) u = __fadd_rn(u, __ldg(a.bias_u + col));
    a.out[(size_t)row * a.n + col] = silu_mul(g, u);
}

// Element sel (0-2) of a kernel-parameter array by selects: a runtime index into the
// parameter space would copy the whole argument struct to local memory.
template <typename P>
__device__ __forceinline__ P pick3(P const (&v)[3], int sel) {
    return sel == 0 ? v[0] : sel == 1 ? v[1] : v[2];
}

// ROPE: x row r of the call, matrix sel, rows ra and ra + d/2 of a head (va, vb before bias)
__device__ __forceinline__ void finish_rope(const PairParams& p, int r, int sel, int ra, float va, float vb) {
    const int half = p.d >> 1, i = ra % p.d;
    const float* bias = pick3(p.bias, sel);
    if (bias) {
        va = __fadd_rn(va, __ldg(bias + ra));
        vb = __fadd_rn(vb, __ldg(bias + ra + half));
    }
    const int tok = p.m0 + r;
    const int seq = tok / p.n_tok, t = tok - seq * p.n_tok;
    const size_t pos = (size_t)p.n_past + t;
    // separately rounded products and sums, as the reference's rope (src/llm.zig:221-238)
    const float c = p.cos_tab[pos * half + i], s = p.sin_tab[pos * half + i];
    const float lo = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
    const float hi = __fadd_rn(__fmul_rn(va, s), __fmul_rn(vb, c));
    if (sel == 0) {
        float* qo = p.q_out + (size_t)tok * p.n_head * p.d + ra;
        qo[0] = lo;
        qo[half] = hi;
    } else {
        float* kt = p.cache_kt + (size_t)seq * p.cache_bs;
        kt[(size_t)ra * p.n_ctx + pos] = lo;
        kt[(size_t)(ra + half) * p.n_ctx + pos] = hi;
    }
}

// ROPE's v rows: bias, then the V cache at the token's position
__device__ __forceinline__ void finish_rope_v(const PairParams& p, int r, int ra, float v) {
    if (p.bias[2]) v = __fadd_rn(v, __ldg(p.bias[2] + ra));
    const int tok = p.m0 + r;
    const int seq = tok / p.n_tok, t = tok - seq * p.n_tok;
    const size_t pos = (size_t)p.n_past + t;
    p.cache_v[(size_t)seq * p.cache_bs + pos * ((size_t)p.n_head_kv * p.d) + ra] = v;
}

// QKV: x row r of the call (window r / n_tok, token r % n_tok), matrix sel, column col
__device__ __forceinline__ void finish_qkv(const PairParams& p, int r, int sel, int col, float v) {
    const float* bias = pick3(p.bias, sel);
    if (bias) v = __fadd_rn(v, __ldg(bias + col));
    if (sel == 0) {
        p.q_out[(size_t)r * p.d + col] = v;
        return;
    }
    const int seq = r / p.n_tok, t = r - seq * p.n_tok;
    float* cache = sel == 1 ? p.cache_kt : p.cache_v;
    cache[(size_t)seq * p.cache_bs + ((size_t)p.n_past + t) * p.d + col] = v;
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_cluster(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, const void* dst, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int c0, int c1) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(map), "r"(c0), "r"(c1) : "memory");
}

// EPI: the epilogue mode. The SiLU pair's tile rows 0-63 are the gate's rows j0.., 64-127
// the up matrix's same rows (tm_w, tm_wu); ROPE and QKV read matrix sel's rows j0.. through
// tm_w, tm_wu or tm_w3. SMALL: the 64-row tile form (Tr).
template <int EPI, bool SMALL>
__global__ void __launch_bounds__(THREADS, 1)
    q8_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wu,
                 const __grid_constant__ CUtensorMap tm_w3, const __grid_constant__ CUtensorMap tm_x, Args a) {
    constexpr bool PAIR = EPI == EPI_SILU;
    constexpr bool SEC = EPI == EPI_ROPE || EPI == EPI_QKV;  // three matrices, one per tile
    using T = Tr<SMALL>;
    constexpr int TN = T::TN, NSR = T::NSR, NSC = T::NSC, NSLOT = T::NSLOT, COLS = T::COLS;
    constexpr uint32_t RAW_X = T::RAW_X, CV_P = T::CV_P, ACC = T::ACC;
    extern __shared__ uint8_t smem_raw[];
    Smem<SMALL>& sm =
        *reinterpret_cast<Smem<SMALL>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rows_w = PAIR ? BM / 2 : BM;               // weight rows of one matrix per tile
    int sel = 0, j0 = blockIdx.x * rows_w;
    if (SEC) {
        const int bx = blockIdx.x;
        sel = bx < a.tiles[0] ? 0 : bx < a.tiles[0] + a.tiles[1] ? 1 : 2;
        j0 = (bx - (sel > 0 ? a.tiles[0] : 0) - (sel > 1 ? a.tiles[1] : 0)) * BM;
    }
    const CUtensorMap* tmw = (!SEC || sel == 0) ? &tm_w : sel == 1 ? &tm_wu : &tm_w3;
    const int r0 = blockIdx.y * TN;
    const int rank = blockIdx.z;                          // = the CTA's rank in its cluster
    const int steps_all = a.k / BK;
    const int s_begin = (int)(((long long)rank * steps_all) / a.ks);
    const int s_end = (int)(((long long)(rank + 1) * steps_all) / a.ks);
    const int steps = s_end - s_begin;
    const int nbk = a.k / 32;                             // Q8 blocks per weight row

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSR; s++) {
            mbar_init(&sm.raw_full[s], 1);
            mbar_init(&sm.raw_empty[s], CONV_THREADS);
        }
        for (int s = 0; s < NSC; s++) {
            mbar_init(&sm.cv_full[s], CONV_THREADS);
            mbar_init(&sm.cv_empty[s], 1);
        }
        for (int s = 0; s < NSLOT; s++) {
            mbar_init(&sm.acc_full[s], 1);
            mbar_init(&sm.acc_empty[s], SCALE_WARPS);
        }
        fence_mbar_init();
    }
    // the weights are constants: warm L2 with this CTA's first steps before waiting for the
    // kernel that wrote x
    if (warp == 0 && lane == 0) {
        prefetch_tmap(tmw);
        prefetch_tmap(&tm_x);
        if (PAIR) prefetch_tmap(&tm_wu);
        for (int i = 0; i < steps && i < 4; i++) {
            tma_prefetch_2d(tmw, (s_begin + i) * BK, j0);
            if (PAIR) tma_prefetch_2d(&tm_wu, (s_begin + i) * BK, j0);
        }
    }
    // TMEM is taken only after the previous kernel has completed and before the next one may
    // start: a CTA of either that shares this SM may hold or wait for TMEM, and this CTA must
    // never hold columns while it waits for a kernel that may be waiting for them.
    const int z = chain_wait();
    a.out += z;
    if (a.bias) a.bias += z;
    if (a.bias_u) a.bias_u += z;
    if (warp == 1) {
        tmem_alloc(&sm.tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    chain_release();
    const uint32_t tmem = sm.tmem_base;

    bool ok = true;
    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < steps; i++) {
                const int rs = i % NSR;
                if (i >= NSR && !(ok = mbar_wait(&sm.raw_empty[rs], ((i / NSR) - 1) & 1, a.err))) break;
                const int kc = (s_begin + i) * BK;
                mbar_arrive_expect_tx(&sm.raw_full[rs], RAW_W + RAW_X);
                tma_load_2d(tmw, &sm.raw_full[rs], sm.raw_w[rs], kc, j0);
                if (PAIR) tma_load_2d(&tm_wu, &sm.raw_full[rs], sm.raw_w[rs] + RAW_W / 2, kc, j0);
                tma_load_2d(&tm_x, &sm.raw_full[rs], sm.raw_x[rs], kc, r0);
                issued = i + 1;
            }
            // copies still in flight land before the CTA's shared memory goes away
            for (int i = issued > NSR ? issued - NSR : 0; i < issued; i++)
                mbar_wait_drain(&sm.raw_full[i % NSR], (i / NSR) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(BM, SMALL ? NP * TN : TN, true, false, false);
            int blk = 0;
            for (int i = 0; ok && i < steps; i++) {
                const int cs = i % NSC;
                if (!(ok = mbar_wait(&sm.cv_full[cs], (i / NSC) & 1, a.err))) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sm.cv_a[cs]);
                const uint32_t b_addr = smem_u32(sm.cv_b[cs]);
                for (int hb = 0; hb < 2; hb++, blk++) {
                    const int slot = blk % NSLOT;
                    if (blk >= NSLOT && !(ok = mbar_wait(&sm.acc_empty[slot], ((blk / NSLOT) - 1) & 1, a.err))) break;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        const uint32_t ko = (uint32_t)(hb * 2 + kk) * 32;  // 16 bf16 = 32 bytes of k
                        if constexpr (SMALL) {
                            // the three pieces as one B operand of 192 rows: their dots side by side
                            mma_f16_ss(tmem + slot * ACC, smem_desc_sw128(a_addr + ko, 16, 1024),
                                       smem_desc_sw128(b_addr + ko, 16, 1024), idesc, kk ? 1u : 0u);
                        } else {
#pragma unroll
                            for (int p = 0; p < NP; p++)
                                mma_f16_ss(tmem + slot * ACC, smem_desc_sw128(a_addr + ko, 16, 1024),
                                           smem_desc_sw128(b_addr + p * CV_P + ko, 16, 1024), idesc,
                                           (kk | p) ? 1u : 0u);
                        }
                    }
                    mma_commit(&sm.acc_full[slot]);
                }
                if (!ok) break;
                mma_commit(&sm.cv_empty[cs]);
            }
            // the last products complete before TMEM is freed
            if (blk > 0) mbar_wait_drain(&sm.acc_full[(blk - 1) % NSLOT], ((blk - 1) / NSLOT) & 1);
        }
    } else if (warp < SCALE_WARP0) {
        // ------------------------------------------------------------ converters
        const int ct = threadIdx.x - 64;                  // 0..255
        for (int i = 0; i < steps; i++) {
            const int rs = i % NSR, cs = i % NSC;
            if (!(ok = mbar_wait_warp(&sm.raw_full[rs], (i / NSR) & 1, a.err))) break;
            if (i >= NSC && !(ok = mbar_wait_warp(&sm.cv_empty[cs], ((i / NSC) - 1) & 1, a.err))) break;
            const uint32_t rw = smem_u32(sm.raw_w[rs]), rx = smem_u32(sm.raw_x[rs]);
            const uint32_t ca = smem_u32(sm.cv_a[cs]), cb = smem_u32(sm.cv_b[cs]);
            // Every shared load of the step is issued before the first conversion, so the
            // thread waits out one load latency per step instead of one per chunk.
            // weights: row r, 16 int8 (chunk c4 of the 64-byte row) -> two 16-byte chunks
            uint4 wv[2];
#pragma unroll
            for (int u = 0; u < 2; u++) wv[u] = ld_shared_v4(rw + ((ct >> 2) + 64 * u) * BK + (ct & 3) * 16);
            // activations: row r, 8 f32 (chunk c8, two 16-byte halves) -> one 16-byte chunk
            // of each piece. Lane map: the 8 lanes of a quarter warp take 4 chunks of row r
            // (half 0 first) and the same 4 chunks of row r + 4 (half 1 first), so their
            // loads fall in 8 distinct bank groups and so do their stores (swizzle r & 7
            // differs in bit 2). Rows past m stay zero once written.
            const int xh = (ct >> 2) & 1, q4 = (ct >> 3) & 3, cw = ct >> 5;
            const int c8 = (ct & 3) + 4 * (q4 & 1);
            const int xr = 4 * xh + (q4 >> 1) + 2 * (cw & 1) + 8 * (cw >> 1);
            uint4 xa[TN / 32], xb[TN / 32];
#pragma unroll
            for (int u = 0; u < TN / 32; u++) {
                const int r = xr + 32 * u;
                if (i >= NSC && r0 + r >= a.m) continue;
                xa[u] = ld_shared_v4(rx + r * (BK * 4) + c8 * 32 + xh * 16);
                xb[u] = ld_shared_v4(rx + r * (BK * 4) + c8 * 32 + (xh ^ 1) * 16);
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int r = (ct >> 2) + 64 * u, c4 = ct & 3;
                const uint4 w = wv[u];
                uint4 o0, o1;
                int8x4_to_bf16(w.x, o0.x, o0.y);
                int8x4_to_bf16(w.y, o0.z, o0.w);
                int8x4_to_bf16(w.z, o1.x, o1.y);
                int8x4_to_bf16(w.w, o1.z, o1.w);
                const int sw = r & 7;
                st_shared_v4(ca + r * 128 + (((2 * c4) ^ sw) << 4), o0);
                st_shared_v4(ca + r * 128 + (((2 * c4 + 1) ^ sw) << 4), o1);
            }
#pragma unroll
            for (int u = 0; u < TN / 32; u++) {
                const int r = xr + 32 * u;
                if (i >= NSC && r0 + r >= a.m) continue;
                const uint4 x0 = xh ? xb[u] : xa[u];
                const uint4 x1 = xh ? xa[u] : xb[u];
                uint4 ph, pm, pl;
                split3(__uint_as_float(x0.x), __uint_as_float(x0.y), ph.x, pm.x, pl.x);
                split3(__uint_as_float(x0.z), __uint_as_float(x0.w), ph.y, pm.y, pl.y);
                split3(__uint_as_float(x1.x), __uint_as_float(x1.y), ph.z, pm.z, pl.z);
                split3(__uint_as_float(x1.z), __uint_as_float(x1.w), ph.w, pm.w, pl.w);
                const uint32_t off = r * 128 + ((c8 ^ (r & 7)) << 4);
                st_shared_v4(cb + off, ph);
                st_shared_v4(cb + CV_P + off, pm);
                st_shared_v4(cb + 2 * CV_P + off, pl);
            }
            // every raw value has been consumed: the stage goes back to the producer before
            // the proxy fence below waits for this thread's stores
            mbar_arrive(&sm.raw_empty[rs]);
            // the tensor core (async proxy) reads what these threads wrote
            fence_proxy_async_smem();
            mbar_arrive(&sm.cv_full[cs]);
        }
    }
    // the producer and MMA warps ran their loops in lane 0 alone: every warp reaches the
    // CTA and cluster barriers below converged
    __syncwarp();

    // ------------------------------------------------------------ scalers and epilogue
    float2 acc2[COLS / 2];                                 // (row 2c, row 2c + 1) of this thread's rows
#pragma unroll
    for (int c = 0; c < COLS / 2; c++) acc2[c] = make_float2(0.f, 0.f);
    const bool scaler = warp >= SCALE_WARP0;
    const int jl = scaler ? (warp & 3) * 32 + lane : 0;   // tile row = TMEM lane
    const int cg = scaler ? (warp - SCALE_WARP0) >> 2 : 0; // which half of the activation rows
    const bool up = PAIR && jl >= BM / 2;
    const int jrow = j0 + (PAIR ? (jl & (BM / 2 - 1)) : jl);  // row of its matrix
    // ROPE / QKV: every matrix has whole 128-row tiles (the launcher checks it)
    const bool row_ok = SEC || jrow < a.n;
    if (scaler) {
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16) + cg * COLS;
        const float* sbase = SEC ? pick3(a.pp.ws, sel) : up ? a.wsu : a.ws;
        const float* srow = sbase + (size_t)(row_ok ? jrow : 0) * nbk;
        const int b0 = s_begin * 2;
        float s_next = row_ok ? __ldg(srow + b0) : 0.f;
        for (int blk = 0; blk < 2 * steps; blk++) {
            const int slot = blk % NSLOT;
            const float s = s_next;
            if (blk + 1 < 2 * steps) s_next = row_ok ? __ldg(srow + b0 + blk + 1) : 0.f;
            if (!(ok = mbar_wait_warp(&sm.acc_full[slot], (blk / NSLOT) & 1, a.err))) break;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < COLS / 16; h++) {
                const float2 s2 = make_float2(s, s);
                if constexpr (SMALL) {
                    // the block dot of each row is (hi + mid) + lo over its three columns
                    uint32_t vh[16], vm[16], vl[16];
                    tmem_ld16(lane_base + slot * ACC + h * 16, vh);
                    tmem_ld16(lane_base + slot * ACC + TN + h * 16, vm);
                    tmem_ld16(lane_base + slot * ACC + 2 * TN + h * 16, vl);
                    tmem_ld_wait();
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const float2 d = __fadd2_rn(
                            __fadd2_rn(make_float2(__uint_as_float(vh[2 * c]), __uint_as_float(vh[2 * c + 1])),
                                       make_float2(__uint_as_float(vm[2 * c]), __uint_as_float(vm[2 * c + 1]))),
                            make_float2(__uint_as_float(vl[2 * c]), __uint_as_float(vl[2 * c + 1])));
                        acc2[h * 8 + c] = __ffma2_rn(s2, d, acc2[h * 8 + c]);
                    }
                } else {
                    uint32_t v[16];
                    tmem_ld16(lane_base + slot * ACC + h * 16, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int c = 0; c < 8; c++)
                        acc2[h * 8 + c] = __ffma2_rn(
                            s2, make_float2(__uint_as_float(v[2 * c]), __uint_as_float(v[2 * c + 1])), acc2[h * 8 + c]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[slot]);
        }
    }

    // the operand ring is free once every MMA has completed (the scalers saw the last one)
    // and every copy has landed; it then holds the partial tile or the pair's exchange
    __syncthreads();
    float acc[COLS];
#pragma unroll
    for (int c = 0; c < COLS / 2; c++) {
        acc[2 * c] = acc2[c].x;
        acc[2 * c + 1] = acc2[c].y;
    }
    float* part = reinterpret_cast<float*>(sm.cv_b[0]);
    const int cbase = cg * COLS;                           // first activation row of this thread
    // ROPE: a head's rows i < d/2 finish the pair (i, i + d/2); the v matrix has no pairs
    const int half = a.pp.d >> 1;
    const bool rope_pairs = EPI == EPI_ROPE && sel != 2;
    const bool second = rope_pairs && (jrow % a.pp.d) >= half;
    if (a.ks == 1) {
        if (scaler) {
            if (EPI == EPI_PLAIN) {
                if (row_ok) {
#pragma unroll
                    for (int c = 0; c < COLS; c++)
                        if (r0 + cbase + c < a.m) finish(a, r0 + cbase + c, jrow, acc[c]);
                }
            } else if (EPI == EPI_QKV) {
#pragma unroll
                for (int c = 0; c < COLS; c++)
                    if (r0 + cbase + c < a.m) finish_qkv(a.pp, r0 + cbase + c, sel, jrow, acc[c]);
            } else if (EPI == EPI_ROPE) {
                if (!rope_pairs) {
#pragma unroll
                    for (int c = 0; c < COLS; c++)
                        if (r0 + cbase + c < a.m) finish_rope_v(a.pp, r0 + cbase + c, jrow, acc[c]);
                } else {
                    // sel is the CTA's: every scaler thread reaches the barrier
                    if (second) {
#pragma unroll
                        for (int c = 0; c < COLS; c++) part[(cbase + c) * PART_LD + jl] = acc[c];
                    }
                    named_sync(1, SCALE_THREADS);
                    if (!second)
#pragma unroll
                        for (int c = 0; c < COLS; c++)
                            if (r0 + cbase + c < a.m)
                                finish_rope(a.pp, r0 + cbase + c, sel, jrow, acc[c], part[(cbase + c) * PART_LD + jl + half]);
                }
            } else {
                if (up) {
#pragma unroll
                    for (int c = 0; c < COLS; c++) part[(cbase + c) * PAIR_LD + (jl - BM / 2)] = acc[c];
                }
                named_sync(1, SCALE_THREADS);
                if (!up && row_ok)
#pragma unroll
                    for (int c = 0; c < COLS; c++)
                        if (r0 + cbase + c < a.m) finish_pair(a, r0 + cbase + c, jrow, acc[c], part[(cbase + c) * PAIR_LD + jl]);
            }
        }
    } else {
        if (scaler) {
#pragma unroll
            for (int c = 0; c < COLS; c++) part[(cbase + c) * PART_LD + jl] = acc[c];
        }
        cluster_sync();
        if (scaler && row_ok) {
            // this CTA's share of the activation rows, summed over the ranks in rank order.
            // The remote loads of 16 / ks rows (all ks ranks each) are issued before the
            // first add, so a batch costs one round trip through the cluster, not one per row
            // (ks is 2, 4 or 8: the batch sizes are compile-time, the arrays registers).
            const int c0 = (rank * TN) / a.ks, c1 = ((rank + 1) * TN) / a.ks;
            // a RoPE pair's first row also sums its partner's column
            const uint32_t partner = (uint32_t)half * 4;
            auto reduce = [&](auto ks_c) {
                constexpr int KS = decltype(ks_c)::value;
                constexpr int RB = 16 / KS;  // rows per batch
                uint32_t base[KS];
#pragma unroll
                for (int rk = 0; rk < KS; rk++) base[rk] = cluster_addr(part + jl, rk);
                for (int cb = c0 + cg; cb < c1 && !second; cb += 2 * RB) {
                    if (r0 + cb >= a.m) break;
                    float p[RB][KS], q[RB][KS];
#pragma unroll
                    for (int u = 0; u < RB; u++) {
                        // rows past the share load a row of it (in bounds) and are not used
                        const int c = min(cb + 2 * u, c1 - 1);
#pragma unroll
                        for (int rk = 0; rk < KS; rk++) {
                            p[u][rk] = ld_cluster(base[rk] + c * PART_LD * 4);
                            q[u][rk] = rope_pairs ? ld_cluster(base[rk] + c * PART_LD * 4 + partner) : 0.f;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < RB; u++) {
                        const int c = cb + 2 * u;
                        if (c >= c1 || r0 + c >= a.m) break;
                        float v = 0.f, vb = 0.f;
#pragma unroll
                        for (int rk = 0; rk < KS; rk++) {
                            v = __fadd_rn(v, p[u][rk]);
                            vb = __fadd_rn(vb, q[u][rk]);
                        }
                        if (EPI == EPI_PLAIN) finish(a, r0 + c, jrow, v);
                        else if (EPI == EPI_QKV) finish_qkv(a.pp, r0 + c, sel, jrow, v);
                        else if (rope_pairs) finish_rope(a.pp, r0 + c, sel, jrow, v, vb);
                        else finish_rope_v(a.pp, r0 + c, jrow, v);
                    }
                }
            };
            if (a.ks == 2) reduce(std::integral_constant<int, 2>{});
            else if (a.ks == 4) reduce(std::integral_constant<int, 4>{});
            else reduce(std::integral_constant<int, 8>{});
        }
        // no CTA leaves while another may still read its partial tile
        cluster_sync();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace q8tc

namespace q8tc {
std::atomic<int> g_enabled{1};
}

namespace {

bool map_2d(CUtensorMap* m, CUtensorMapDataType ty, const void* base, uint64_t inner, uint64_t outer,
            uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    return fn(m, ty, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

}  // namespace

namespace {

// How many clusters of cs CTAs (1 x 1 x cs) of kernel variant `variant` can be resident at
// once on device dev (the occupancy API's answer, cached); 0 when the query fails.
int max_clusters(int dev, int variant, const void* kern, size_t smem, int cs) {
    static std::mutex mu;
    static int cache[64][8][4] = {};
    const int li = cs == 2 ? 1 : cs == 4 ? 2 : cs == 8 ? 3 : 0;
    std::lock_guard<std::mutex> lk(mu);
    int& slot = cache[dev][variant][li];
    if (slot == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, 1, (unsigned)cs);
        cfg.blockDim = dim3(q8tc::THREADS);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 1;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = (unsigned)cs;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            n = 0;
        }
        slot = n > 0 ? n : -1;
    }
    return slot > 0 ? slot : 0;
}

// One launch of the tensor-core kernel for x [m][k] against the weight tiles of the mode
// (PLAIN / SILU: n rows of wq (and wu); ROPE / QKV: the three matrices of pp, rows[i] each).
// Returns 1 when the shape is not covered (the caller runs the CUDA-core kernel), 0 after a
// launch, -1 on a launch failure.
int tc_launch(int epi, const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias,
              size_t n, int mode, const int8_t* wu, const float* su, const float* bu, const PairParams* pp,
              const size_t* rows, float* out, int sm_count, cudaStream_t st) {
    using namespace q8tc;
    const bool pair = epi == EPI_SILU, sec = epi == EPI_ROPE || epi == EPI_QKV;
    const int use = q8tc::g_enabled.load(std::memory_order_relaxed);
    if (!use) return 1;
    if (m < 16 || n == 0 || k == 0 || k % BK) return 1;
    // by size (the default): at up to 64 rows a short k over a small matrix is faster on the
    // CUDA-core kernel, which has no fixed cost of TMEM, barriers and a cluster reduction
    // (measured at 32 rows: 512 x 512 6.7 against 10.4 us, 2048 x 512 8.5 against 12.4,
    // 896 x 896 at 64 rows 12.4 against 14.4; k 1536 and up, or more weights, favour the
    // tensor cores: 512 x 2048 12.6 against 14.5, 51864 x 512 37 against 90)
    if (use == 1 && m <= 64 && k <= 1024) {
        const size_t w_rows = sec ? rows[0] + rows[1] + rows[2] : pair ? 2 * n : n;
        if (w_rows * k <= (size_t)1310720) return 1;
    }
    if (((uintptr_t)x & 15) || ((uintptr_t)wq & 15) || (pair && ((uintptr_t)wu & 15))) return 1;
    if (m > (1u << 30) || n > (1u << 30) || k > (1u << 30)) return 1;
    if (pair && mode != LIN_STORE) return 1;
    if (sec)
        for (int i = 0; i < 3; i++)
            if (rows[i] == 0 || rows[i] % BM || !pp->wq[i] || ((uintptr_t)pp->wq[i] & 15)) return 1;
    // up to 64 rows the small tile form (pieces along N), else the large one
    const bool small = m <= 64;
    const int tn = small ? Tr<true>::TN : Tr<false>::TN;
    const int rows_w = pair ? BM / 2 : BM;
    const size_t tiles_n = sec ? (rows[0] + rows[1] + rows[2]) / BM : (n + rows_w - 1) / rows_w;
    const size_t tiles_m = (m + tn - 1) / tn;
    if (tiles_n > 0x7fffffff || tiles_m > 65535) return 1;

    CUtensorMap mw, mwu, mw3, mx;
    if (sec) {
        if (!map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, pp->wq[0], k, rows[0], k, BK, BM) ||
            !map_2d(&mwu, CU_TENSOR_MAP_DATA_TYPE_UINT8, pp->wq[1], k, rows[1], k, BK, BM) ||
            !map_2d(&mw3, CU_TENSOR_MAP_DATA_TYPE_UINT8, pp->wq[2], k, rows[2], k, BK, BM))
            return -1;
    } else {
        if (!map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, k, n, k, BK, rows_w)) return -1;
        if (pair && !map_2d(&mwu, CU_TENSOR_MAP_DATA_TYPE_UINT8, wu, k, n, k, BK, rows_w)) return -1;
        if (!pair) mwu = mw;
        mw3 = mw;
    }
    if (!map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, x, k, m, k * 4, BK, (uint32_t)tn)) return -1;

    Args a{};
    a.m = (int)m;
    a.n = (int)n;
    a.k = (int)k;
    a.mode = mode;
    a.ws = ws;
    a.wsu = su;
    a.bias = bias;
    a.bias_u = bu;
    a.out = out;
    a.err = capi::current_err_word();
    if (sec) {
        a.pp = *pp;
        for (int i = 0; i < 3; i++) a.tiles[i] = (int)(rows[i] / BM);
    }

    static std::mutex mu;
    static bool attr_set[64][8] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    const int variant = epi * 2 + (small ? 1 : 0);
    using Kern = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, Args);
    static const Kern kerns[8] = {q8_tc_kernel<EPI_PLAIN, false>, q8_tc_kernel<EPI_PLAIN, true>,
                                  q8_tc_kernel<EPI_SILU, false>,  q8_tc_kernel<EPI_SILU, true>,
                                  q8_tc_kernel<EPI_ROPE, false>,  q8_tc_kernel<EPI_ROPE, true>,
                                  q8_tc_kernel<EPI_QKV, false>,   q8_tc_kernel<EPI_QKV, true>};
    const Kern kern = kerns[variant];
    const size_t smem = small ? smem_bytes<true>() : smem_bytes<false>();
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[dev][variant]) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return -1;
            attr_set[dev][variant] = true;
        }
    }
    // k splits (powers of two, at most 8, at least two k steps each) while the doubled grid
    // still fits in one wave (one CTA per SM) and its clusters can all be resident at once
    // (a cluster lies within one GPC, so fewer clusters of 4 or 8 fit than SMs / size): a
    // second, mostly empty wave costs more than the longer k ranges; the pair keeps whole k
    // ranges
    const size_t steps = k / BK;
    int ks = 1;
    while (!pair && ks < MAX_KS && tiles_n * tiles_m * (size_t)(2 * ks) <= (size_t)std::max(1, sm_count) &&
           steps / (2 * ks) >= 2 &&
           tiles_n * tiles_m <= (size_t)max_clusters(dev, variant, (const void*)kern, smem, 2 * ks))
        ks *= 2;
    a.ks = ks;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)ks);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
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
    return cudaLaunchKernelEx(&cfg, kern, mw, mwu, mw3, mx, a) == cudaSuccess ? 0 : -1;
}

}  // namespace

// The tensor-core Q8 product when it applies: returns 1 (not taken: the caller runs the
// CUDA-core kernel) for shapes it does not cover, 0 after a launch, -1 on a launch failure.
// wu/su/bu non-null: the SiLU pair (out = silu(x . Wg^T + bg) * (x . Wu^T + bu)).
int q8_tc_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias, size_t n,
                 int mode, const int8_t* wu, const float* su, const float* bu, float* out, int sm_count,
                 cudaStream_t st) {
    return tc_launch(wu ? q8tc::EPI_SILU : q8tc::EPI_PLAIN, x, m, k, wq, ws, bias, n, mode, wu, su, bu, nullptr,
                     nullptr, out, sm_count, st);
}

// The Qwen2 RoPE pair (q8_pair_launch's PAIR_ROPE) on the tensor cores: q, k and v of
// p.n_head / p.n_head_kv heads of p.d rows, rows of each matrix a multiple of 128.
int q8_tc_rope_launch(const PairParams& p, int sm_count, cudaStream_t st) {
    const size_t rows[3] = {(size_t)p.n_head * p.d, (size_t)p.n_head_kv * p.d, (size_t)p.n_head_kv * p.d};
    if (p.d <= 0 || q8tc::BM % p.d) return 1;
    return tc_launch(q8tc::EPI_ROPE, p.x, (size_t)p.m, (size_t)p.k, p.wq[0], p.ws[0], nullptr,
                     rows[0] + rows[1] + rows[2], LIN_STORE, nullptr, nullptr, nullptr, &p, rows, nullptr, sm_count,
                     st);
}

// The Whisper decoder's q/k/v product (q8_gemm_qkv_launch's PE_QKV) on the tensor cores:
// three matrices of p.d rows, p.d a multiple of 128.
int q8_tc_qkv_launch(const PairParams& p, int sm_count, cudaStream_t st) {
    const size_t rows[3] = {(size_t)p.d, (size_t)p.d, (size_t)p.d};
    return tc_launch(q8tc::EPI_QKV, p.x, (size_t)p.m, (size_t)p.k, p.wq[0], p.ws[0], nullptr, 3 * (size_t)p.d,
                     LIN_STORE, nullptr, nullptr, nullptr, &p, rows, nullptr, sm_count, st);
}

}  // namespace zwg

extern "C" ZWG_API int zwg_q8_tensor_cores(int enable) {
    if (enable < 0) return zwg::q8tc::g_enabled.load();
    return zwg::q8tc::g_enabled.exchange(enable >= 2 ? 2 : enable ? 1 : 0);
}
