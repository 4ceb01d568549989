// C-ABI entry points of the Whisper decoder step around the attention (include/zwgpu.h):
// Decoder.forward and setAudio (src/decoder.zig:151-206) as LayerNorm, Q8 projections with
// their biases and epilogues (residual add, GELU), the token + position embedding and the
// tied logits, around the state's self- and cross-attention (zwg_dec_step_attn, state.cu).
// Arguments are checked as the reference's asserts would; the calls only launch work on the
// caller's stream.
#include <cuda_runtime.h>

#include "../../include/zwgpu.h"
#include "api_internal.h"
#include "kernels.h"

using namespace zwg::capi;

namespace {

constexpr float kLnEps = 1e-5f;  // ops.layerNorm's epsilon (src/ops.zig:393-396)

bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }
bool al4(const void* p) { return ((uintptr_t)p & 3) == 0; }

int check_mat(const zwg_q8_mat& m, const char* name) {
    if (!m.q || !m.scales) return fail("%s: null Q8 matrix", name);
    if (!al16(m.q) || !al4(m.scales)) return fail("%s: int8 data must be 16-byte aligned, scales 4-byte", name);
    return ZWG_OK;
}

int check_vec16(const float* v, const char* name) {
    if (!v || !al16(v)) return fail("%s: null or not 16-byte aligned", name);
    return ZWG_OK;
}

int check_layer(const zwg_dec_layer_weights& L) {
    int rc = ZWG_OK;
    const zwg_q8_mat* mats[] = {&L.q, &L.k, &L.v, &L.o, &L.cq, &L.ck, &L.cv, &L.co, &L.mlp0, &L.mlp1};
    const char* names[] = {"q", "k", "v", "o", "cq", "ck", "cv", "co", "mlp0", "mlp1"};
    for (int i = 0; i < 10 && !rc; i++) rc = check_mat(*mats[i], names[i]);
    const float* norms[] = {L.attn_ln_w, L.attn_ln_b, L.cross_ln_w, L.cross_ln_b, L.mlp_ln_w, L.mlp_ln_b};
    for (int i = 0; i < 6 && !rc; i++) rc = check_vec16(norms[i], "layer norm weights");
    const float* biases[] = {L.q_b, L.v_b, L.o_b, L.cq_b, L.cv_b, L.co_b, L.mlp0_b, L.mlp1_b};
    for (int i = 0; i < 8 && !rc; i++)
        if (!biases[i] || !al4(biases[i])) rc = fail("decoder biases: null or not 4-byte aligned");
    return rc;
}

size_t round_floats(size_t f) { return (f + 63) & ~(size_t)63; }  // 256-byte steps

struct Scratch {
    float *h, *q, *k, *v, *attn, *hid;  // [rows][n_state] each, hid [rows][4 n_state]
    size_t bytes;
};

Scratch carve(void* base, size_t rows, size_t ns) {
    Scratch s;
    float* p = static_cast<float*>(base);
    const size_t a = round_floats(rows * ns);
    s.h = p;
    s.q = p + a;
    s.k = p + 2 * a;
    s.v = p + 3 * a;
    s.attn = p + 4 * a;
    s.hid = p + 5 * a;
    s.bytes = (5 * a + round_floats(rows * 4 * ns)) * sizeof(float);
    return s;
}

int lin(const float* x, size_t m, size_t k, const zwg_q8_mat& w, const float* bias, size_t n, int mode, float* out,
        cudaStream_t s, const char* what) {
    if (zwg::q8_linear_launch(x, m, k, w.q, w.scales, bias, n, mode, out, s)) return cuda_fail(what, cudaGetLastError());
    return ZWG_OK;
}

int ln(const float* x, size_t stride, size_t m, size_t n, const float* w, const float* b, float* out, size_t ostride,
       cudaStream_t s) {
    if (zwg::layer_norm_launch(x, stride, m, n, w, b, kLnEps, out, ostride, s))
        return cuda_fail("layer_norm launch", cudaGetLastError());
    return ZWG_OK;
}

}  // namespace

extern "C" {

int zwg_layer_norm(const float* x, size_t m, size_t n, const float* w, const float* b, float eps, float* out,
                   void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (m == 0) return ZWG_OK;
    if (!x || !w || !b || !out) return fail("layer_norm: null buffer");
    if (n == 0 || n % 4) return fail("layer_norm: n = %zu must be a positive multiple of 4", n);
    if (!al16(x) || !al16(w) || !al16(b) || !al16(out)) return fail("layer_norm: buffers must be 16-byte aligned");
    if (m >= (1u << 31) || n >= (1u << 30)) return fail("layer_norm: too large");
    if (zwg::layer_norm_launch(x, n, m, n, w, b, eps, out, n, (cudaStream_t)stream))
        return cuda_fail("layer_norm launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_linear_q8_gelu(const float* x, size_t m, size_t k, const int8_t* q, const float* scales, const float* bias,
                       size_t n, float* out, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (k == 0 || k % 32) return fail("linear_q8_gelu: k = %zu must be a positive multiple of 32", k);
    if (m == 0 || n == 0) return ZWG_OK;
    if (!x || !q || !scales || !out) return fail("linear_q8_gelu: null buffer");
    if (!al16(x) || !al16(q)) return fail("linear_q8_gelu: x and q must be 16-byte aligned");
    if (!al4(scales) || !al4(out) || !al4(bias)) return fail("linear_q8_gelu: f32 buffers must be 4-byte aligned");
    if (n >= (1u << 30) || k >= (1u << 30) || m >= (1u << 30)) return fail("linear_q8_gelu: matrix too large");
    if (zwg::q8_linear_launch(x, m, k, q, scales, bias, n, zwg::LIN_GELU, out, (cudaStream_t)stream))
        return cuda_fail("linear_q8_gelu launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_dec_set_audio_q8(zwg_dec_state* st, const zwg_dec_weights* w, size_t window, const float* enc, void* stream) {
    if (!st || !w || !w->layers) return fail("dec_set_audio_q8: null state or weights");
    if (window >= st->n_batch) return fail("dec_set_audio_q8: window %zu >= n_batch %zu", window, st->n_batch);
    if (!enc || !al16(enc)) return fail("dec_set_audio_q8: enc null or not 16-byte aligned");
    Ctx* c = ctx_for(st->device);
    if (!c) return ZWG_ERROR;
    const size_t ns = st->n_state, na = st->n_audio_ctx;
    if (ns % 32) return fail("dec_set_audio_q8: n_state must be a multiple of 32");
    const cudaStream_t s = (cudaStream_t)stream;
    for (size_t l = 0; l < st->n_layer; l++) {
        const zwg_dec_layer_weights& L = w->layers[l];
        int rc = check_mat(L.ck, "ck");
        if (!rc) rc = check_mat(L.cv, "cv");
        if (!rc && (!L.cv_b || !al4(L.cv_b))) rc = fail("dec_set_audio_q8: cv_b null or misaligned");
        // src/decoder.zig:154-155
        if (!rc) rc = lin(enc, na, ns, L.ck, nullptr, ns, zwg::LIN_STORE, st->cross_k[l] + window * na * ns, s, "ck launch");
        if (!rc) rc = lin(enc, na, ns, L.cv, L.cv_b, ns, zwg::LIN_STORE, st->cross_v[l] + window * na * ns, s, "cv launch");
        if (rc) return rc;
    }
    return ZWG_OK;
}

size_t zwg_dec_scratch_bytes(const zwg_dec_state* st, size_t n) {
    if (!st) return 0;
    return carve(nullptr, st->n_batch * n, st->n_state).bytes;
}

int zwg_dec_forward_q8(zwg_dec_state* st, const zwg_dec_weights* w, const int32_t* tokens, size_t n_past, size_t n,
                       float* x, float* logits, void* scratch, size_t scratch_bytes, void* stream) {
    if (!st || !w || !w->layers) return fail("dec_forward_q8: null state or weights");
    if (n == 0) return ZWG_OK;
    if (n_past + n > st->n_text_ctx) return fail("dec_forward_q8: context full (%zu + %zu > %zu)", n_past, n, st->n_text_ctx);
    Ctx* c = ctx_for(st->device);
    if (!c) return ZWG_ERROR;
    const size_t ns = st->n_state, nb = st->n_batch, M = nb * n;
    if (ns % 32) return fail("dec_forward_q8: n_state must be a multiple of 32");
    if (!tokens || !x || !logits || !scratch) return fail("dec_forward_q8: null buffer");
    if (!al4(tokens) || !al16(x) || !al4(logits) || ((uintptr_t)scratch & 255))
        return fail("dec_forward_q8: tokens and logits 4-byte, x 16-byte, scratch 256-byte aligned");
    if (!w->n_vocab || w->n_vocab >= (1u << 30) || M >= (1u << 30)) return fail("dec_forward_q8: bad sizes");
    int rc = check_mat(w->te, "te");
    if (!rc) rc = check_vec16(w->ln_w, "ln_w");
    if (!rc) rc = check_vec16(w->ln_b, "ln_b");
    if (!rc && (!w->pe || !al4(w->pe))) rc = fail("dec_forward_q8: pe null or misaligned");
    for (size_t l = 0; l < st->n_layer && !rc; l++) rc = check_layer(w->layers[l]);
    if (rc) return rc;
    const Scratch sc = carve(scratch, M, ns);
    if (scratch_bytes < sc.bytes) return fail("dec_forward_q8: scratch %zu bytes, %zu needed", scratch_bytes, sc.bytes);
    const cudaStream_t s = (cudaStream_t)stream;

    // src/decoder.zig:172-176: token row + position row
    if (zwg::embed_q8_launch(tokens, M, w->te.q, w->te.scales, w->n_vocab, ns, w->pe, n_past, n, x, c->err, s))
        return cuda_fail("embed launch", cudaGetLastError());
    for (size_t l = 0; l < st->n_layer; l++) {
        const zwg_dec_layer_weights& L = w->layers[l];
        // masked self-attention over the cache (src/decoder.zig:180-186)
        if ((rc = ln(x, ns, M, ns, L.attn_ln_w, L.attn_ln_b, sc.h, ns, s))) return rc;
        if (M >= 16) {
            // q, k and v in one tiled product whose epilogue appends k and v to the caches
            zwg::PairParams p{};
            p.x = sc.h;
            p.m = (int)M;
            p.k = (int)ns;
            p.wq[0] = L.q.q; p.wq[1] = L.k.q; p.wq[2] = L.v.q;
            p.ws[0] = L.q.scales; p.ws[1] = L.k.scales; p.ws[2] = L.v.scales;
            p.bias[0] = L.q_b; p.bias[2] = L.v_b;
            p.d = (int)ns;
            p.n_tok = (int)n;
            p.n_past = (int)n_past;
            p.q_out = sc.q;
            p.cache_kt = st->self_k[l];
            p.cache_v = st->self_v[l];
            p.cache_bs = st->n_text_ctx * ns;
            if (zwg::q8_gemm_qkv_launch(p, c->sm_count, s)) return cuda_fail("qkv launch", cudaGetLastError());
            rc = zwg_dec_step_attn(st, l, ZWG_DEC_SELF, sc.q, nullptr, nullptr, n_past, n, sc.attn, stream);
        } else {
            if ((rc = lin(sc.h, M, ns, L.q, L.q_b, ns, zwg::LIN_STORE, sc.q, s, "q launch"))) return rc;
            if ((rc = lin(sc.h, M, ns, L.k, nullptr, ns, zwg::LIN_STORE, sc.k, s, "k launch"))) return rc;
            if ((rc = lin(sc.h, M, ns, L.v, L.v_b, ns, zwg::LIN_STORE, sc.v, s, "v launch"))) return rc;
            rc = zwg_dec_step_attn(st, l, ZWG_DEC_SELF, sc.q, sc.k, sc.v, n_past, n, sc.attn, stream);
        }
        if (rc) return rc;
        if ((rc = lin(sc.attn, M, ns, L.o, L.o_b, ns, zwg::LIN_ADD, x, s, "o launch"))) return rc;
        // cross-attention over the audio (src/decoder.zig:188-193)
        if ((rc = ln(x, ns, M, ns, L.cross_ln_w, L.cross_ln_b, sc.h, ns, s))) return rc;
        if ((rc = lin(sc.h, M, ns, L.cq, L.cq_b, ns, zwg::LIN_STORE, sc.q, s, "cq launch"))) return rc;
        if ((rc = zwg_dec_step_attn(st, l, ZWG_DEC_CROSS, sc.q, nullptr, nullptr, 0, n, sc.attn, stream))) return rc;
        if ((rc = lin(sc.attn, M, ns, L.co, L.co_b, ns, zwg::LIN_ADD, x, s, "co launch"))) return rc;
        // mlp (src/decoder.zig:195-200)
        if ((rc = ln(x, ns, M, ns, L.mlp_ln_w, L.mlp_ln_b, sc.h, ns, s))) return rc;
        if ((rc = lin(sc.h, M, ns, L.mlp0, L.mlp0_b, 4 * ns, zwg::LIN_GELU, sc.hid, s, "mlp0 launch"))) return rc;
        if ((rc = lin(sc.hid, M, 4 * ns, L.mlp1, L.mlp1_b, ns, zwg::LIN_ADD, x, s, "mlp1 launch"))) return rc;
    }
    // src/decoder.zig:203-205: the last token of each window, tied logits
    if ((rc = ln(x + (n - 1) * ns, n * ns, nb, ns, w->ln_w, w->ln_b, sc.h, ns, s))) return rc;
    return lin(sc.h, nb, ns, w->te, nullptr, w->n_vocab, zwg::LIN_STORE, logits, s, "logits launch");
}

}  // extern "C"
