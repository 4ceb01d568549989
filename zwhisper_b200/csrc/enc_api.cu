// C-ABI entry points of the Whisper encoder on the device (include/zwgpu.h): Encoder.forward
// (src/encoder.zig:118-179) as the conv front-end and the pre-norm blocks around the tcgen05
// attention, every product an f16 GEMM on the tensor cores (gemm_tc.cu), and the single GEMM
// entry point those are built from. The calls only launch work on the caller's stream.
//
// Data flow per call (n_windows windows of T = 2 n_ctx mel frames, n_state = ns):
//   mel -> rows16 [w][T + 2][n_mels] f16 (frame t in row t + 1, zero rows around)
//   conv1: rows t-1, t, t+1 as one operand row (stride n_mels, 3 n_mels wide)
//          -> gelu(. conv1_w^T + b) -> x1 [w][T + 1][ns] f16, row 0 zero (frame -1)
//   conv2: x1 rows 2t-1, 2t, 2t+1 (stride 2 ns, 3 ns wide) -> gelu(. conv2_w^T + b) + pos
//          -> x [w][n_ctx][ns] f32 (the output buffer holds the residual stream)
//   per block: h = LN(x) f16; qkv = h . w_qkv^T + b_qkv (bf16 [w][n_ctx][3 ns]);
//          a = attention(q, k, v) f16; x += a . w_o^T + b_o; h = LN(x);
//          hid = gelu(h . w_mlp0^T + b) f16; x += hid . w_mlp2^T + b
//   out = LN_post(x), in place.
#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/zwgpu.h"
#include "api_internal.h"
#include "kernels.h"

using namespace zwg::capi;

namespace {

constexpr float kLnEps = 1e-5f;  // ops.layerNorm's epsilon (src/ops.zig:393-396)

bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }
size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

struct EncScratch {
    uint16_t* rows16;  // mel rows, then (aliased) qkv
    uint16_t* qkv;
    uint16_t* x1;      // conv1 output, then (aliased) the MLP hidden rows
    uint16_t* hid;
    uint16_t* h;       // LayerNorm output
    uint16_t* attn;    // attention output
    size_t bytes;
};

// Region sizes: [0] mel rows / qkv, [1] x1 / hidden rows, [2] h, [3] attention output.
void region_bytes(const zwg_enc_weights* w, size_t nw, size_t r[4]) {
    const size_t ns = w->n_state, T = 2 * w->n_ctx;
    const size_t rows_b = nw * (T + 2) * w->n_mels * 2, qkv_b = nw * w->n_ctx * 3 * ns * 2;
    const size_t x1_b = nw * (T + 1) * ns * 2, hid_b = nw * w->n_ctx * 4 * ns * 2;
    r[0] = round256(std::max(rows_b, qkv_b));
    r[1] = round256(std::max(x1_b, hid_b));
    r[2] = r[3] = round256(nw * w->n_ctx * ns * 2);
}

EncScratch carve(void* base, const zwg_enc_weights* w, size_t nw) {
    size_t r[4];
    region_bytes(w, nw, r);
    EncScratch s;
    char* p = static_cast<char*>(base);
    s.rows16 = s.qkv = reinterpret_cast<uint16_t*>(p);
    s.x1 = s.hid = reinterpret_cast<uint16_t*>(p + r[0]);
    s.h = reinterpret_cast<uint16_t*>(p + r[0] + r[1]);
    s.attn = reinterpret_cast<uint16_t*>(p + r[0] + r[1] + r[2]);
    s.bytes = r[0] + r[1] + r[2] + r[3];
    return s;
}

int check_weights(const zwg_enc_weights* w) {
    if (!w) return fail("encoder: null weights");
    const size_t ns = w->n_state;
    if (ns % 128 || ns < 128 || ns > 1024 || w->n_head * 64 != ns)
        return fail("encoder: n_state %zu must be a multiple of 128 up to 1024 with 64-wide heads (n_head %zu)", ns,
                    w->n_head);
    if (!w->n_mels || w->n_mels % 8 || !w->n_ctx || w->n_ctx > (1u << 20) || !w->layers)
        return fail("encoder: bad sizes (n_mels %zu, n_ctx %zu)", w->n_mels, w->n_ctx);
    const void* ptrs[] = {w->conv1_w, w->conv1_b, w->conv2_w, w->conv2_b, w->pos, w->ln_post_w, w->ln_post_b};
    for (const void* p : ptrs)
        if (!p || !al16(p)) return fail("encoder: a weight pointer is null or not 16-byte aligned");
    for (size_t l = 0; l < w->n_layer; l++) {
        const zwg_enc_layer_weights& L = w->layers[l];
        const void* lp[] = {L.attn_ln_w, L.attn_ln_b, L.w_qkv, L.b_qkv, L.w_o, L.b_o,
                            L.mlp_ln_w, L.mlp_ln_b, L.w_mlp0, L.b_mlp0, L.w_mlp2, L.b_mlp2};
        for (const void* p : lp)
            if (!p || !al16(p)) return fail("encoder layer %zu: a weight pointer is null or not 16-byte aligned", l);
    }
    return ZWG_OK;
}

zwg::GemmParams gemm(const uint16_t* a, size_t lda, size_t a_bs, const uint16_t* wt, size_t ldw, size_t M, size_t N,
                     size_t K, size_t nb) {
    zwg::GemmParams p{};
    p.a = a;
    p.lda = lda;
    p.a_bs = a_bs;
    p.w = wt;
    p.ldw = ldw;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.n_batch = (int)nb;
    return p;
}

int run_gemm(Ctx* c, const zwg::GemmParams& p, const char* what, cudaStream_t st) {
    if (!zwg::gemm_f16_supported(p)) return fail("%s: shape or alignment not supported by the f16 GEMM", what);
    if (zwg::gemm_f16_launch(p, c->sm_count, c->err, st)) return cuda_fail(what, cudaGetLastError());
    return ZWG_OK;
}

}  // namespace

extern "C" {

size_t zwg_mel_frames(size_t n_samples) { return zwg::mel_frames(n_samples); }

size_t zwg_mel_scratch_bytes(void) { return zwg::mel_scratch_bytes(); }

int zwg_log_mel(const float* samples, size_t n_samples, const float* filters, size_t n_mel, float* out, void* scratch,
                size_t scratch_bytes, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (!samples || !filters || !out || !scratch) return fail("log_mel: null pointer");
    if (n_samples == 0 || n_samples > (size_t)1 << 40) return fail("log_mel: bad sample count %zu", n_samples);
    if (n_mel == 0 || n_mel > 1024) return fail("log_mel: bad n_mel %zu", n_mel);
    if (scratch_bytes < zwg::mel_scratch_bytes() || !al16(scratch))
        return fail("log_mel: scratch must be 16-byte aligned and at least %zu bytes", zwg::mel_scratch_bytes());
    if (zwg::log_mel_launch(samples, n_samples, filters, (int)n_mel, out, scratch, c->sm_count, (cudaStream_t)stream))
        return cuda_fail("log_mel launch", cudaGetLastError());
    return ZWG_OK;
}

size_t zwg_enc_scratch_bytes(const zwg_enc_weights* w, size_t n_windows) {
    if (!w || !w->n_state || !w->n_ctx) return 0;
    size_t r[4];
    region_bytes(w, n_windows, r);
    return r[0] + r[1] + r[2] + r[3];
}

int zwg_gemm_f16(const uint16_t* a, size_t lda, size_t a_bs, const uint16_t* w, size_t ldw, size_t M, size_t N,
                 size_t K, size_t n_batch, const float* bias, int gelu, const float* addend, size_t ld_add,
                 int accumulate, void* out, int out_type, size_t ld_out, size_t out_bs, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (M == 0 || N == 0 || n_batch == 0) return ZWG_OK;
    if (!a || !w || !out) return fail("gemm_f16: null pointer");
    if (M > (1u << 30) || N > (1u << 30) || K == 0 || K > (1u << 30) || n_batch > 65535)
        return fail("gemm_f16: bad sizes (M %zu, N %zu, K %zu, batch %zu)", M, N, K, n_batch);
    zwg::GemmParams p = gemm(a, lda, a_bs, w, ldw, M, N, K, n_batch);
    p.out_type = out_type;
    p.gelu = gelu != 0;
    p.accumulate = accumulate != 0;
    p.e.bias = bias;
    p.e.addend = addend;
    p.e.ld_add = ld_add;
    p.e.out = out;
    p.e.ld_out = ld_out;
    p.e.out_bs = out_bs ? out_bs : ld_out * M;
    return run_gemm(c, p, "gemm_f16", (cudaStream_t)stream);
}

int zwg_enc_forward_f16(const zwg_enc_weights* w, const float* mel, size_t n_len, const int32_t* offsets,
                        size_t n_windows, float* out, void* scratch, size_t scratch_bytes, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    int rc = check_weights(w);
    if (rc) return rc;
    if (n_windows == 0) return ZWG_OK;
    if (n_windows > 65535) return fail("encoder: at most 65535 windows per call");
    if (!mel || !out || !scratch) return fail("encoder: null mel, out or scratch");
    if (!al16(out) || !al16(scratch) || !al16(mel)) return fail("encoder: mel, out and scratch must be 16-byte aligned");
    const size_t ns = w->n_state, n_ctx = w->n_ctx, T = 2 * n_ctx, nw = n_windows, nm = w->n_mels;
    const EncScratch s = carve(scratch, w, nw);
    if (scratch_bytes < s.bytes) return fail("encoder: scratch too small: %zu < %zu bytes", scratch_bytes, s.bytes);
    cudaStream_t st = (cudaStream_t)stream;

    // mel frames as f16 rows with a zero row on each side
    if (zwg::mel_rows_launch(mel, (int)nm, n_len, offsets, (int)nw, (int)T, s.rows16, st))
        return cuda_fail("encoder mel rows", cudaGetLastError());
    // conv1 (src/encoder.zig:125-140): operand row t = rows t-1, t, t+1; output row t at x1 row t + 1
    {
        zwg::GemmParams p = gemm(s.rows16, nm, (T + 2) * nm, w->conv1_w, 3 * nm, T, ns, 3 * nm, nw);
        p.out_type = zwg::GEMM_OUT_F16;
        p.gelu = true;
        p.e.bias = w->conv1_b;
        p.e.out = s.x1 + ns;
        p.e.ld_out = ns;
        p.e.out_bs = (T + 1) * ns;
        if ((rc = run_gemm(c, p, "encoder conv1", st))) return rc;
    }
    // frame -1 of the second convolution's input is zero
    cudaError_t e = cudaMemset2DAsync(s.x1, (T + 1) * ns * 2, 0, ns * 2, nw, st);
    if (e != cudaSuccess) return cuda_fail("encoder conv padding", e);
    // conv2 (stride 2, src/encoder.zig:141-150) + positional embedding: operand row t = x1
    // rows 2t-1, 2t, 2t+1 (buffer rows 2t .. 2t+2)
    {
        zwg::GemmParams p = gemm(s.x1, 2 * ns, (T + 1) * ns, w->conv2_w, 3 * ns, n_ctx, ns, 3 * ns, nw);
        p.out_type = zwg::GEMM_OUT_F32;
        p.gelu = true;
        p.e.bias = w->conv2_b;
        p.e.addend = w->pos;
        p.e.ld_add = ns;
        p.e.out = out;
        p.e.ld_out = ns;
        p.e.out_bs = n_ctx * ns;
        if ((rc = run_gemm(c, p, "encoder conv2", st))) return rc;
    }
    const size_t rows = nw * n_ctx;
    for (size_t l = 0; l < w->n_layer; l++) {
        const zwg_enc_layer_weights& L = w->layers[l];
        // attention block (src/encoder.zig:153-168)
        if (zwg::layer_norm_rows_launch(out, rows, (int)ns, L.attn_ln_w, L.attn_ln_b, kLnEps, s.h, true, st))
            return cuda_fail("encoder attn_ln", cudaGetLastError());
        {
            zwg::GemmParams p = gemm(s.h, ns, n_ctx * ns, L.w_qkv, ns, n_ctx, 3 * ns, ns, nw);
            p.out_type = zwg::GEMM_OUT_BF16;
            p.e.bias = L.b_qkv;
            p.e.out = s.qkv;
            p.e.ld_out = 3 * ns;
            p.e.out_bs = n_ctx * 3 * ns;
            if ((rc = run_gemm(c, p, "encoder qkv", st))) return rc;
        }
        {
            zwg::EncTcParams p{s.qkv, s.qkv + ns, s.qkv + 2 * ns, reinterpret_cast<float*>(s.attn), (int)nw,
                               (int)n_ctx, (int)w->n_head, c->err};
            p.ld_qkv = 3 * ns;
            p.out_f16 = 1;
            if (zwg::enc_tc_launch(p, st)) return cuda_fail("encoder attention", cudaGetLastError());
        }
        {
            zwg::GemmParams p = gemm(s.attn, ns, n_ctx * ns, L.w_o, ns, n_ctx, ns, ns, nw);
            p.out_type = zwg::GEMM_OUT_F32;
            p.accumulate = true;
            p.e.bias = L.b_o;
            p.e.out = out;
            p.e.ld_out = ns;
            p.e.out_bs = n_ctx * ns;
            if ((rc = run_gemm(c, p, "encoder attn out", st))) return rc;
        }
        // MLP block (src/encoder.zig:170-176)
        if (zwg::layer_norm_rows_launch(out, rows, (int)ns, L.mlp_ln_w, L.mlp_ln_b, kLnEps, s.h, true, st))
            return cuda_fail("encoder mlp_ln", cudaGetLastError());
        {
            zwg::GemmParams p = gemm(s.h, ns, n_ctx * ns, L.w_mlp0, ns, n_ctx, 4 * ns, ns, nw);
            p.out_type = zwg::GEMM_OUT_F16;
            p.gelu = true;
            p.e.bias = L.b_mlp0;
            p.e.out = s.hid;
            p.e.ld_out = 4 * ns;
            p.e.out_bs = n_ctx * 4 * ns;
            if ((rc = run_gemm(c, p, "encoder mlp0", st))) return rc;
        }
        {
            zwg::GemmParams p = gemm(s.hid, 4 * ns, n_ctx * 4 * ns, L.w_mlp2, 4 * ns, n_ctx, ns, 4 * ns, nw);
            p.out_type = zwg::GEMM_OUT_F32;
            p.accumulate = true;
            p.e.bias = L.b_mlp2;
            p.e.out = out;
            p.e.ld_out = ns;
            p.e.out_bs = n_ctx * ns;
            if ((rc = run_gemm(c, p, "encoder mlp2", st))) return rc;
        }
    }
    // ln_post (src/encoder.zig:178), in place
    if (zwg::layer_norm_rows_launch(out, rows, (int)ns, w->ln_post_w, w->ln_post_b, kLnEps, out, false, st))
        return cuda_fail("encoder ln_post", cudaGetLastError());
    return ZWG_OK;
}

}  // extern "C"
