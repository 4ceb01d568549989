/*
 * C restatement of the reference attention (src/ops.zig:464-605, src/gemm.zig:139-186).
 *
 * TEST INFRASTRUCTURE ONLY: the timed CPU baseline ("port") and a cross-check of the
 * numpy restatement. The product never links or calls this file.
 *
 * Same algorithm and task split as the reference:
 *   - K -> KT[hk][d][n_kv_pad] per kv head, zero padded (AttnJob.transpose, ops.zig:505-515),
 *     skipped when the caller keeps keys transposed (kt_stride, ops.zig:488-491);
 *   - n_head x ceil(n_q/64) tasks (ops.zig:584-589), each:
 *       S = Q_h . KT by the broadcast-FMA block kernel (pvBlock, gemm.zig:139-186),
 *       scale 1/sqrt(d), softmax over the causal limit with the Cephes exp
 *       (expVec, ops.zig:177-209; softmaxRow, ops.zig:442-462), zero the tail,
 *       O = S . V_h (pvBlock again);
 *   - tasks are pulled dynamically by the worker threads like Pool.parallelFor
 *     (ops.zig:126-145); OpenMP's dynamic schedule plays that role here.
 * Vector width: 16 lanes with AVX-512, 8 with AVX2 (gemm.zig:15-23).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#include <omp.h>

#if defined(__AVX512F__)
#define VW 16
#else
#define VW 8
#endif

typedef float vf __attribute__((vector_size(VW * 4), aligned(4)));
typedef int32_t vi __attribute__((vector_size(VW * 4), aligned(4)));

#define QBLOCK 64

typedef struct zwref_shape {
    size_t n_q, n_kv, n_head, n_head_kv, d;
    size_t q_stride, kv_stride, out_stride;
    int causal;
    size_t kt_stride; /* 0: keys are rows [n_kv][kv_stride]; else [n_head_kv][d][kt_stride] */
} zwref_shape;

static inline vf vsplat(float x) { return (vf){0} + x; }
static inline vf vload(const float* p) { vf v; memcpy(&v, p, sizeof v); return v; }
static inline void vstore(float* p, vf v) { memcpy(p, &v, sizeof v); }
static inline vf vsel(vi m, vf a, vf b) {
    vi ai, bi;
    memcpy(&ai, &a, sizeof a);
    memcpy(&bi, &b, sizeof b);
    vi r = (ai & m) | (bi & ~m);
    vf o;
    memcpy(&o, &r, sizeof o);
    return o;
}
static inline vf vmin(vf a, vf b) { return vsel(a < b, a, b); }
static inline vf vmax(vf a, vf b) { return vsel(a > b, a, b); }
/* floor for |x| < 2^23: truncate, then step down where truncation went up */
static inline vf vfloor(vf x) {
    vf t = __builtin_convertvector(__builtin_convertvector(x, vi), vf);
    return vsel(t > x, t - vsplat(1.0f), t);
}

/* expVec (ops.zig:177-209): Cephes range reduction and degree-5 polynomial. */
static inline vf exp_vec(vf x) {
    const vf lo = vsplat(-87.3f), hi = vsplat(88.3f);
    x = vmax(vmin(x, hi), lo);
    vf fx = vfloor(x * vsplat(1.44269504088896341f) + vsplat(0.5f));
    vf r = x - fx * vsplat(0.693359375f);
    r = r - fx * vsplat(-2.12194440e-4f);
    vf y = vsplat(1.9875691500e-4f) * r + vsplat(1.3981999507e-3f);
    y = y * r + vsplat(8.3334519073e-3f);
    y = y * r + vsplat(4.1665795894e-2f);
    y = y * r + vsplat(1.6666665459e-1f);
    y = y * r + vsplat(5.0000001201e-1f);
    vf r2 = r * r;
    y = y * r2 + r;
    y = y + vsplat(1.0f);
    vi e = (__builtin_convertvector(fx, vi) + 127) << 23;
    vf sc;
    memcpy(&sc, &e, sizeof sc);
    return y * sc;
}

/* softmaxRow (ops.zig:442-462) */
static void softmax_row(float* x, size_t n) {
    if (n == 0) return;
    vf mxv = vsplat(-INFINITY);
    size_t i = 0;
    for (; i + VW <= n; i += VW) mxv = vmax(mxv, vload(x + i));
    float mx = -INFINITY;
    for (int l = 0; l < VW; l++) mx = mxv[l] > mx ? mxv[l] : mx;
    for (; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    vf mv = vsplat(mx), sv = vsplat(0.f);
    i = 0;
    for (; i + VW <= n; i += VW) {
        vf e = exp_vec(vload(x + i) - mv);
        vstore(x + i, e);
        sv += e;
    }
    float sum = 0.f;
    for (int l = 0; l < VW; l++) sum += sv[l];
    for (; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    /* scale (ops.zig:223-231) */
    const float inv = 1.0f / sum;
    const vf iv = vsplat(inv);
    for (i = 0; i + VW <= n; i += VW) vstore(x + i, vload(x + i) * iv);
    for (; i < n; i++) x[i] *= inv;
}

/* pvBlock (gemm.zig:139-186): C[m][d] = P[m][t] . V[t][d], d % VW == 0.
 * Four query rows at a time with up to four vectors of d each in registers. */
#define PV_TILE(W)                                                                     \
    do {                                                                               \
        vf acc[4][W];                                                                  \
        for (int r = 0; r < 4; r++)                                                    \
            for (int q = 0; q < W; q++) acc[r][q] = vsplat(0.f);                       \
        for (size_t tt = 0; tt < t; tt++) {                                            \
            const float* vrow = v + tt * ldv + dv * VW;                                \
            vf p0 = vsplat(p[(i + 0) * ldp + tt]), p1 = vsplat(p[(i + 1) * ldp + tt]); \
            vf p2 = vsplat(p[(i + 2) * ldp + tt]), p3 = vsplat(p[(i + 3) * ldp + tt]); \
            _Pragma("GCC unroll 4") for (int q = 0; q < W; q++) {                      \
                vf vv = vload(vrow + q * VW);                                          \
                acc[0][q] += p0 * vv;                                                  \
                acc[1][q] += p1 * vv;                                                  \
                acc[2][q] += p2 * vv;                                                  \
                acc[3][q] += p3 * vv;                                                  \
            }                                                                          \
        }                                                                              \
        for (int r = 0; r < 4; r++)                                                    \
            for (int q = 0; q < W; q++) vstore(c + (i + r) * ldc + (dv + q) * VW, acc[r][q]); \
    } while (0)

static void pv_block(const float* p, size_t ldp, const float* v, size_t ldv, float* c, size_t ldc,
                     size_t m, size_t t, size_t d) {
    size_t nd = d / VW, i = 0;
    for (; i + 4 <= m; i += 4) {
        for (size_t dv = 0; dv < nd; dv += 4) {
            size_t w = nd - dv < 4 ? nd - dv : 4;
            switch (w) {
                case 4: PV_TILE(4); break;
                case 3: PV_TILE(3); break;
                case 2: PV_TILE(2); break;
                default: PV_TILE(1); break;
            }
        }
    }
    for (; i < m; i++) {
        float* out = c + i * ldc;
        memset(out, 0, d * sizeof(float));
        for (size_t tt = 0; tt < t; tt++) {
            vf s = vsplat(p[i * ldp + tt]);
            const float* vrow = v + tt * ldv;
            for (size_t q = 0; q < d; q += VW) vstore(out + q, s * vload(vrow + q) + vload(out + q));
        }
    }
}

size_t zwref_vector_width(void) { return VW; }

/* attentionScratchEx / attentionScratchKT (ops.zig:545-560), in floats. */
size_t zwref_scratch_floats(const zwref_shape* sh) {
    size_t n_kv_pad = sh->kt_stride ? sh->kt_stride : (sh->n_kv + VW - 1) / VW * VW;
    size_t n_qblocks = (sh->n_q + QBLOCK - 1) / QBLOCK;
    size_t kt_len = sh->kt_stride ? 0 : sh->n_head_kv * sh->d * n_kv_pad;
    return kt_len + sh->n_head * n_qblocks * QBLOCK * n_kv_pad;
}

/* attentionEx (ops.zig:562-590). Returns 0, or 2 on a shape the reference asserts against. */
int zwref_attention_ex(const zwref_shape* sh, const float* q, const float* k, const float* v,
                       float* scratch, float* out, int n_threads) {
    if (sh->d % VW || sh->n_head_kv == 0 || sh->n_head % sh->n_head_kv) return 2;
    if (sh->causal && sh->n_kv < sh->n_q) return 2;
    if (sh->kt_stride && (sh->kt_stride % VW || sh->kt_stride < sh->n_kv)) return 2;
    const size_t d = sh->d;
    const size_t n_kv_pad = sh->kt_stride ? sh->kt_stride : (sh->n_kv + VW - 1) / VW * VW;
    const size_t n_qblocks = (sh->n_q + QBLOCK - 1) / QBLOCK;
    const size_t kt_len = sh->kt_stride ? 0 : sh->n_head_kv * d * n_kv_pad;
    const float* kt = sh->kt_stride ? k : scratch;
    float* scores = scratch + kt_len;
    if (n_threads <= 0) n_threads = omp_get_max_threads();
    if (!sh->kt_stride) {
        float* ktw = scratch;
#pragma omp parallel for num_threads(n_threads) schedule(dynamic, 1)
        for (size_t h = 0; h < sh->n_head_kv; h++) {
            float* dst = ktw + h * d * n_kv_pad;
            for (size_t t = 0; t < sh->n_kv; t++) {
                const float* src = k + t * sh->kv_stride + h * d;
                for (size_t p = 0; p < d; p++) dst[p * n_kv_pad + t] = src[p];
            }
            for (size_t p = 0; p < d; p++)
                for (size_t t = sh->n_kv; t < n_kv_pad; t++) dst[p * n_kv_pad + t] = 0.f;
        }
    }
    const size_t n_tasks = sh->n_head * n_qblocks;
    const size_t group = sh->n_head / sh->n_head_kv;
    const float scl = 1.0f / sqrtf((float)d);
#pragma omp parallel for num_threads(n_threads) schedule(dynamic, 1)
    for (size_t task = 0; task < n_tasks; task++) {
        size_t h = task / n_qblocks, hk = h / group, qb = task % n_qblocks;
        size_t q0 = qb * QBLOCK, q1 = q0 + QBLOCK < sh->n_q ? q0 + QBLOCK : sh->n_q, m = q1 - q0;
        float* sc = scores + task * QBLOCK * n_kv_pad;
        const float* kth = kt + hk * d * n_kv_pad;
        size_t cols = (sh->n_kv + VW - 1) / VW * VW;
        pv_block(q + q0 * sh->q_stride + h * d, sh->q_stride, kth, n_kv_pad, sc, n_kv_pad, m, d, cols);
        for (size_t i = 0; i < m; i++) {
            float* row = sc + i * n_kv_pad;
            size_t limit = sh->causal ? sh->n_kv - sh->n_q + q0 + i + 1 : sh->n_kv;
            size_t t = 0;
            for (; t + VW <= limit; t += VW) vstore(row + t, vload(row + t) * vsplat(scl));
            for (; t < limit; t++) row[t] *= scl;
            softmax_row(row, limit);
            for (t = limit; t < cols; t++) row[t] = 0.f;
        }
        pv_block(sc, n_kv_pad, v + hk * d, sh->kv_stride, out + q0 * sh->out_stride + h * d,
                 sh->out_stride, m, sh->n_kv, d);
    }
    return 0;
}
