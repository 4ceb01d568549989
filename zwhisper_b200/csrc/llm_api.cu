// C-ABI entry points of the Qwen2 decode step around the attention (include/zwgpu.h):
// Model.forward (src/llm.zig:169-216) as norms, fused Q8 projections and the attention of
// state.cu, plus the greedy sampler (src/llm.zig:268-273, 313-321). Every call checks its
// arguments the way the reference's asserts and slice bounds would, then only launches
// kernels on the caller's stream: no allocation, no synchronization.
#include <cuda_runtime.h>

#include "../../include/zwgpu.h"
#include "api_internal.h"
#include "kernels.h"

using namespace zwg::capi;

namespace {

bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }
bool al4(const void* p) { return ((uintptr_t)p & 3) == 0; }

int check_q8(const zwg_q8_mat& m, const char* name) {
    if (!m.q || !m.scales) return fail("%s: null Q8 matrix", name);
    if (!al16(m.q) || !al4(m.scales)) return fail("%s: int8 data must be 16-byte aligned, scales 4-byte", name);
    return ZWG_OK;
}

size_t round_floats(size_t f) { return (f + 63) & ~(size_t)63; }  // 256-byte steps

struct Scratch {
    float* h;     // [M][n_embd] normed hidden states
    float* q;     // [M][n_embd] rotated queries
    float* attn;  // [M][n_embd] attention output
    float* g;     // [M][n_ff] silu(gate) * up
    size_t bytes;
};

Scratch carve(void* base, size_t rows, size_t ne, size_t n_ff) {
    Scratch s;
    float* p = static_cast<float*>(base);
    const size_t a = round_floats(rows * ne), b = round_floats(rows * n_ff);
    s.h = p;
    s.q = p + a;
    s.attn = p + 2 * a;
    s.g = p + 3 * a;
    s.bytes = (3 * a + b) * sizeof(float);
    return s;
}

// Shared checks of a state call: returns the context or nullptr with the error set.
Ctx* state_call(const zwg_llm_state* st, size_t layer, size_t n_past, size_t n, const char* what) {
    if (!st || layer >= st->n_layer) {
        fail("%s: bad state or layer", what);
        return nullptr;
    }
    if (n_past + n > st->n_ctx) {
        fail("%s: context full (%zu + %zu > %zu)", what, n_past, n, st->n_ctx);
        return nullptr;
    }
    return ctx_for(st->device);
}

int check_weights(const zwg_llm_state* st, const zwg_llm_weights* w, const char* what) {
    if (!w || !w->layers) return fail("%s: null weights", what);
    const size_t ne = w->n_embd;
    if (ne != st->n_head * st->d) return fail("%s: n_embd %zu != n_head * d = %zu", what, ne, st->n_head * st->d);
    if (ne % 32 || !w->n_ff || w->n_ff % 32) return fail("%s: n_embd and n_ff must be multiples of 32", what);
    if (ne >= (1u << 30) || w->n_ff >= (1u << 30)) return fail("%s: model too large", what);
    return ZWG_OK;
}

int check_layer(const zwg_llm_layer_weights& L, const char* what) {
    int rc = check_q8(L.wq, "wq");
    if (!rc) rc = check_q8(L.wk, "wk");
    if (!rc) rc = check_q8(L.wv, "wv");
    if (!rc) rc = check_q8(L.wo, "wo");
    if (!rc) rc = check_q8(L.w_gate, "w_gate");
    if (!rc) rc = check_q8(L.w_up, "w_up");
    if (!rc) rc = check_q8(L.w_down, "w_down");
    if (rc) return rc;
    if (!L.attn_norm || !L.ffn_norm) return fail("%s: null norm weights", what);
    if (!al16(L.attn_norm) || !al16(L.ffn_norm)) return fail("%s: norm weights must be 16-byte aligned", what);
    if (!al4(L.bq) || !al4(L.bk) || !al4(L.bv)) return fail("%s: biases must be 4-byte aligned", what);
    return ZWG_OK;
}

int qkv(zwg_llm_state* st, size_t layer, const float* x, const zwg_llm_layer_weights& L, size_t n_past, size_t n,
        float* q_out, cudaStream_t s) {
    zwg::PairParams p{};
    p.x = x;
    p.m = (int)(st->n_batch * n);
    p.k = (int)(st->n_head * st->d);
    p.m0 = 0;
    p.wq[0] = L.wq.q; p.wq[1] = L.wk.q; p.wq[2] = L.wv.q;
    p.ws[0] = L.wq.scales; p.ws[1] = L.wk.scales; p.ws[2] = L.wv.scales;
    p.bias[0] = L.bq; p.bias[1] = L.bk; p.bias[2] = L.bv;
    p.n_pairs = (int)((st->n_head + 2 * st->n_head_kv) * (st->d / 2));
    p.n_head = (int)st->n_head;
    p.n_head_kv = (int)st->n_head_kv;
    p.d = (int)st->d;
    p.n_tok = (int)n;
    p.n_past = (int)n_past;
    p.n_ctx = (int)st->n_ctx;
    p.cos_tab = st->cos_tab;
    p.sin_tab = st->sin_tab;
    p.q_out = q_out;
    p.cache_kt = st->cache_kt[layer];
    p.cache_v = st->cache_v[layer];
    p.cache_bs = st->n_head_kv * st->d * st->n_ctx;
    if (zwg::q8_pair_launch(p, zwg::PAIR_ROPE, s)) return cuda_fail("qkv launch", cudaGetLastError());
    return ZWG_OK;
}

int layer_body(zwg_llm_state* st, size_t layer, const zwg_llm_weights* w, float* x, size_t n_past, size_t n,
               const Scratch& sc, cudaStream_t s) {
    const zwg_llm_layer_weights& L = w->layers[layer];
    int rc = check_layer(L, "llm_layer_q8");
    if (rc) return rc;
    const size_t M = st->n_batch * n, ne = w->n_embd, n_ff = w->n_ff;
    // src/llm.zig:178-190
    if (zwg::rms_norm_launch(x, ne, M, ne, L.attn_norm, w->eps, sc.h, ne, s)) return cuda_fail("rms_norm launch", cudaGetLastError());
    rc = qkv(st, layer, sc.h, L, n_past, n, sc.q, s);
    if (rc) return rc;
    // src/llm.zig:191-202
    rc = llm_attn(st, layer, sc.q, n_past, n, sc.attn, s);
    if (rc) return rc;
    // src/llm.zig:203-204
    if (zwg::q8_linear_launch(sc.attn, M, ne, L.wo.q, L.wo.scales, nullptr, ne, zwg::LIN_ADD, x, s))
        return cuda_fail("wo launch", cudaGetLastError());
    // src/llm.zig:206-210
    if (zwg::rms_norm_launch(x, ne, M, ne, L.ffn_norm, w->eps, sc.h, ne, s)) return cuda_fail("rms_norm launch", cudaGetLastError());
    zwg::PairParams p{};
    p.x = sc.h;
    p.m = (int)M;
    p.k = (int)ne;
    p.wq[0] = L.w_gate.q; p.wq[1] = L.w_up.q;
    p.ws[0] = L.w_gate.scales; p.ws[1] = L.w_up.scales;
    p.n_pairs = (int)n_ff;
    p.out = sc.g;
    if (zwg::q8_pair_launch(p, zwg::PAIR_SILU, s)) return cuda_fail("gate/up launch", cudaGetLastError());
    if (zwg::q8_linear_launch(sc.g, M, n_ff, L.w_down.q, L.w_down.scales, nullptr, ne, zwg::LIN_ADD, x, s))
        return cuda_fail("w_down launch", cudaGetLastError());
    return ZWG_OK;
}

}  // namespace

extern "C" {

int zwg_rms_norm(const float* x, size_t m, size_t n, const float* w, float eps, float* out, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (m == 0) return ZWG_OK;
    if (!x || !w || !out) return fail("rms_norm: null buffer");
    if (n == 0 || n % 4) return fail("rms_norm: n = %zu must be a positive multiple of 4", n);
    if (!al16(x) || !al16(w) || !al16(out)) return fail("rms_norm: buffers must be 16-byte aligned");
    if (m >= (1u << 31) || n >= (1u << 30)) return fail("rms_norm: too large");
    if (zwg::rms_norm_launch(x, n, m, n, w, eps, out, n, (cudaStream_t)stream)) return cuda_fail("rms_norm launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_linear_q8_add(const float* x, size_t m, size_t k, const int8_t* q, const float* scales, size_t n, float* out,
                      void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (k == 0 || k % 32) return fail("linear_q8_add: k = %zu must be a positive multiple of 32", k);
    if (m == 0 || n == 0) return ZWG_OK;
    if (!x || !q || !scales || !out) return fail("linear_q8_add: null buffer");
    if (!al16(x) || !al16(q)) return fail("linear_q8_add: x and q must be 16-byte aligned");
    if (!al4(scales) || !al4(out)) return fail("linear_q8_add: f32 buffers must be 4-byte aligned");
    if (n >= (1u << 30) || k >= (1u << 30) || m >= (1u << 30)) return fail("linear_q8_add: matrix too large");
    if (zwg::q8_linear_launch(x, m, k, q, scales, nullptr, n, zwg::LIN_ADD, out, (cudaStream_t)stream))
        return cuda_fail("linear_q8_add launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_linear_q8_silu_mul(const float* x, size_t m, size_t k, const int8_t* gate_q, const float* gate_scales,
                           const int8_t* up_q, const float* up_scales, size_t n, float* out, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (k == 0 || k % 32) return fail("linear_q8_silu_mul: k = %zu must be a positive multiple of 32", k);
    if (m == 0 || n == 0) return ZWG_OK;
    if (!x || !gate_q || !gate_scales || !up_q || !up_scales || !out) return fail("linear_q8_silu_mul: null buffer");
    if (!al16(x) || !al16(gate_q) || !al16(up_q)) return fail("linear_q8_silu_mul: x and q must be 16-byte aligned");
    if (!al4(gate_scales) || !al4(up_scales) || !al4(out)) return fail("linear_q8_silu_mul: f32 buffers must be 4-byte aligned");
    if (n >= (1u << 30) || k >= (1u << 30) || m >= (1u << 30)) return fail("linear_q8_silu_mul: matrix too large");
    zwg::PairParams p{};
    p.x = x;
    p.m = (int)m;
    p.k = (int)k;
    p.wq[0] = gate_q; p.wq[1] = up_q;
    p.ws[0] = gate_scales; p.ws[1] = up_scales;
    p.n_pairs = (int)n;
    p.out = out;
    if (zwg::q8_pair_launch(p, zwg::PAIR_SILU, (cudaStream_t)stream)) return cuda_fail("silu_mul launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_embed_q8(const int32_t* tokens, size_t m, const int8_t* q, const float* scales, size_t n_vocab, size_t k,
                 float* out, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (k == 0 || k % 32) return fail("embed_q8: k = %zu must be a positive multiple of 32", k);
    if (m == 0) return ZWG_OK;
    if (!tokens || !q || !scales || !out) return fail("embed_q8: null buffer");
    if (!al4(tokens) || !al4(scales) || !al4(out)) return fail("embed_q8: 4-byte alignment required");
    if (m >= (1u << 31) || n_vocab >= (1u << 31) || k >= (1u << 30)) return fail("embed_q8: too large");
    if (zwg::embed_q8_launch(tokens, m, q, scales, n_vocab, k, nullptr, 0, 1, out, c->err, (cudaStream_t)stream))
        return cuda_fail("embed_q8 launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_llm_greedy(float* logits, size_t m, size_t n_vocab, const int32_t* recent, size_t recent_stride,
                   size_t n_recent, size_t window, float penalty, int32_t* out, size_t out_stride, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (m == 0) return ZWG_OK;
    if (!logits || !out || n_vocab == 0) return fail("llm_greedy: null buffer or empty vocabulary");
    if (n_recent && !recent) return fail("llm_greedy: null recent tokens");
    if (n_recent > recent_stride && m > 1) return fail("llm_greedy: n_recent > recent_stride");
    if (m >= (1u << 31) || n_vocab >= (1u << 31) || n_recent >= (1u << 31)) return fail("llm_greedy: too large");
    if (!al4(logits) || !al4(out) || !al4(recent)) return fail("llm_greedy: 4-byte alignment required");
    const size_t win = window < n_recent ? window : n_recent;
    if (zwg::greedy_launch(logits, m, n_vocab, recent, recent_stride, n_recent, win, penalty, out, out_stride, c->err,
                           (cudaStream_t)stream))
        return cuda_fail("llm_greedy launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_llm_qkv_q8(zwg_llm_state* st, size_t layer, const float* x, const zwg_llm_layer_weights* w, size_t n_past,
                   size_t n, float* q_out, void* stream) {
    Ctx* c = state_call(st, layer, n_past, n, "llm_qkv_q8");
    if (!c) return ZWG_ERROR;
    if (n == 0) return ZWG_OK;
    if (!x || !w || !q_out) return fail("llm_qkv_q8: null buffer");
    const size_t ne = st->n_head * st->d;
    if (ne % 32) return fail("llm_qkv_q8: n_head * d = %zu must be a multiple of 32", ne);
    if (!al16(x) || !al4(q_out)) return fail("llm_qkv_q8: x must be 16-byte aligned, q_out 4-byte");
    int rc = check_q8(w->wq, "wq");
    if (!rc) rc = check_q8(w->wk, "wk");
    if (!rc) rc = check_q8(w->wv, "wv");
    if (rc) return rc;
    if (!al4(w->bq) || !al4(w->bk) || !al4(w->bv)) return fail("llm_qkv_q8: biases must be 4-byte aligned");
    if (st->n_batch * n >= (1u << 30)) return fail("llm_qkv_q8: too many rows");
    return qkv(st, layer, x, *w, n_past, n, q_out, (cudaStream_t)stream);
}

size_t zwg_llm_scratch_bytes(const zwg_llm_state* st, size_t n, size_t n_ff) {
    if (!st) return 0;
    const size_t rows = st->n_batch * n;
    return carve(nullptr, rows, st->n_head * st->d, n_ff).bytes;
}

int zwg_llm_layer_q8(zwg_llm_state* st, size_t layer, const zwg_llm_weights* w, float* x, size_t n_past, size_t n,
                     void* scratch, size_t scratch_bytes, void* stream) {
    Ctx* c = state_call(st, layer, n_past, n, "llm_layer_q8");
    if (!c) return ZWG_ERROR;
    if (n == 0) return ZWG_OK;
    int rc = check_weights(st, w, "llm_layer_q8");
    if (rc) return rc;
    if (!x || !scratch) return fail("llm_layer_q8: null buffer");
    if (!al16(x) || ((uintptr_t)scratch & 255)) return fail("llm_layer_q8: x 16-byte, scratch 256-byte aligned");
    if (st->n_batch * n >= (1u << 30)) return fail("llm_layer_q8: too many rows");
    const Scratch sc = carve(scratch, st->n_batch * n, w->n_embd, w->n_ff);
    if (scratch_bytes < sc.bytes) return fail("llm_layer_q8: scratch %zu bytes, %zu needed", scratch_bytes, sc.bytes);
    return layer_body(st, layer, w, x, n_past, n, sc, (cudaStream_t)stream);
}

int zwg_llm_forward_q8(zwg_llm_state* st, const zwg_llm_weights* w, const int32_t* tokens, size_t n_past, size_t n,
                       float* x, float* logits, void* scratch, size_t scratch_bytes, void* stream) {
    Ctx* c = state_call(st, 0, n_past, n, "llm_forward_q8");
    if (!c) return ZWG_ERROR;
    if (n == 0) return ZWG_OK;
    int rc = check_weights(st, w, "llm_forward_q8");
    if (rc) return rc;
    if (!tokens || !x || !logits || !scratch) return fail("llm_forward_q8: null buffer");
    if (!al16(x) || ((uintptr_t)scratch & 255) || !al4(tokens) || !al4(logits))
        return fail("llm_forward_q8: x 16-byte, scratch 256-byte, tokens and logits 4-byte aligned");
    rc = check_q8(w->embd, "embd");
    if (!rc) rc = check_q8(w->output, "output");
    if (rc) return rc;
    if (!w->output_norm || !al16(w->output_norm)) return fail("llm_forward_q8: output_norm null or not 16-byte aligned");
    if (!w->n_vocab || w->n_vocab >= (1u << 30)) return fail("llm_forward_q8: bad n_vocab");
    const size_t M = st->n_batch * n, ne = w->n_embd;
    if (M >= (1u << 30)) return fail("llm_forward_q8: too many rows");
    const Scratch sc = carve(scratch, M, ne, w->n_ff);
    if (scratch_bytes < sc.bytes) return fail("llm_forward_q8: scratch %zu bytes, %zu needed", scratch_bytes, sc.bytes);
    const cudaStream_t s = (cudaStream_t)stream;
    // src/llm.zig:175
    if (zwg::embed_q8_launch(tokens, M, w->embd.q, w->embd.scales, w->n_vocab, ne, nullptr, 0, 1, x, c->err, s))
        return cuda_fail("embed launch", cudaGetLastError());
    for (size_t l = 0; l < st->n_layer; l++) {
        rc = layer_body(st, l, w, x, n_past, n, sc, s);
        if (rc) return rc;
    }
    // src/llm.zig:212-215: the last token of each sequence
    if (zwg::rms_norm_launch(x + (n - 1) * ne, n * ne, st->n_batch, ne, w->output_norm, w->eps, sc.h, ne, s))
        return cuda_fail("rms_norm launch", cudaGetLastError());
    if (zwg::q8_linear_launch(sc.h, st->n_batch, ne, w->output.q, w->output.scales, nullptr, w->n_vocab, zwg::LIN_STORE,
                              logits, s))
        return cuda_fail("logits launch", cudaGetLastError());
    return ZWG_OK;
}

}  // extern "C"
