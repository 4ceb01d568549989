// Library-owned device state for a GPU-resident caller: the Whisper decoder's self and
// cross K/V (src/decoder.zig:39-42, 127-130, 150-156, 166-191) and the Qwen2 LLM's
// transposed key cache, value cache and RoPE tables (src/llm.zig:27-28, 124-137, 168-202),
// each for n_batch windows or sequences. The attention itself runs through the same
// dispatch as zwg_attention_dev (api.cu); this file only owns buffers and turns the
// reference's per-layer calls into batched calls over them.
#include <cuda_runtime.h>

#include <cmath>
#include <vector>

#include "../../include/zwgpu.h"
#include "api_internal.h"
#include "kernels.h"

using namespace zwg::capi;

namespace {

void free_all(std::vector<float*>& v) {
    for (float* p : v)
        if (p) cudaFree(p);
    v.clear();
}

int alloc_layers(std::vector<float*>& v, size_t n_layer, size_t floats, bool zero) {
    v.assign(n_layer, nullptr);
    for (size_t l = 0; l < n_layer; l++) {
        cudaError_t e = cudaMalloc(&v[l], std::max<size_t>(floats, 1) * sizeof(float));
        if (e == cudaSuccess && zero) e = cudaMemset(v[l], 0, floats * sizeof(float));
        if (e != cudaSuccess) return cuda_fail("state allocation", e);
    }
    return ZWG_OK;
}


zwg_attn_shape mha(size_t n_q, size_t n_kv, size_t n_state, size_t n_head, bool causal) {
    return zwg_attn_shape{n_q, n_kv, n_head, n_head, n_state / n_head, n_state, n_state, n_state, causal ? 1 : 0, 0};
}

// Grow the state's workspace to what this call needs (sized for the worst case at
// creation, so this only allocates for shapes beyond it).
int ensure_ws(DevBuf& ws, const zwg_attn_shape* sh, size_t n_batch, int sm_count) {
    const size_t need = workspace_bytes(sh, n_batch, sm_count);
    if (need > ws.cap && !ws.ensure(need)) return fail("workspace allocation of %zu bytes failed", need);
    return ZWG_OK;
}

}  // namespace

Ctx* zwg::capi::ctx_for(int device) {
    Ctx* c = cur();
    if (c && c->device != device) {
        fail("state belongs to device %d, the calling thread is bound to device %d", device, c->device);
        return nullptr;
    }
    return c;
}

int zwg::capi::llm_attn(zwg_llm_state* st, size_t layer, const float* q, size_t n_past, size_t n, float* out,
                        void* stream) {
    if (!st || layer >= st->n_layer) return fail("llm attention: bad state or layer");
    if (n == 0) return ZWG_OK;
    if (!q || !out) return fail("llm attention: null q/out");
    if (n_past + n > st->n_ctx) return fail("llm attention: context full (%zu + %zu > %zu)", n_past, n, st->n_ctx);
    Ctx* c = ctx_for(st->device);
    if (!c) return ZWG_ERROR;
    const size_t H = st->n_head, Hkv = st->n_head_kv, d = st->d, n_ctx = st->n_ctx;
    // the reference's call (src/llm.zig:191-202), over every sequence of the batch
    zwg_attn_shape sh{n, n_past + n, H, Hkv, d, H * d, Hkv * d, H * d, 1, n_ctx};
    zwg_batch b{st->n_batch, n * H * d, Hkv * d * n_ctx, n_ctx * Hkv * d, n * H * d};
    int rc = check_shape(&sh);
    if (!rc) rc = ensure_ws(st->ws, &sh, st->n_batch, c->sm_count);
    if (rc) return rc;
    int* tk = st->tickets.get(c, st->n_batch * Hkv, (cudaStream_t)stream);
    if (!tk) return fail("llm attention: ticket buffer");
    return run_dev(c, &sh, &b, q, st->cache_kt[layer], st->cache_v[layer], out, st->ws.ptr, st->ws.cap,
                   (cudaStream_t)stream, tk);
}

extern "C" {

// ---- Whisper decoder ----------------------------------------------------------------------

int zwg_dec_state_create(size_t n_layer, size_t n_batch, size_t n_state, size_t n_head, size_t n_text_ctx,
                         size_t n_audio_ctx, zwg_dec_state** out) {
    if (!out) return fail("null output pointer");
    *out = nullptr;
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (!n_layer || !n_batch || !n_head || !n_text_ctx || !n_audio_ctx || n_state % n_head || (n_state / n_head) % 4)
        return fail("decoder state: bad sizes (n_state %zu, n_head %zu)", n_state, n_head);
    zwg_dec_state* st = new zwg_dec_state();
    st->device = c->device;
    st->n_layer = n_layer;
    st->n_batch = n_batch;
    st->n_state = n_state;
    st->n_head = n_head;
    st->n_text_ctx = n_text_ctx;
    st->n_audio_ctx = n_audio_ctx;
    int rc = alloc_layers(st->self_k, n_layer, n_batch * n_text_ctx * n_state, false);
    if (!rc) rc = alloc_layers(st->self_v, n_layer, n_batch * n_text_ctx * n_state, false);
    if (!rc) rc = alloc_layers(st->cross_k, n_layer, n_batch * n_audio_ctx * n_state, true);
    if (!rc) rc = alloc_layers(st->cross_v, n_layer, n_batch * n_audio_ctx * n_state, true);
    if (!rc) {
        // worst case of a step: 8 query rows (the decode kernel's limit) over either cache
        const size_t rows = std::min<size_t>(8, n_text_ctx);
        zwg_attn_shape s1 = mha(rows, n_text_ctx, n_state, n_head, true);
        zwg_attn_shape s2 = mha(rows, n_audio_ctx, n_state, n_head, false);
        rc = ensure_ws(st->ws, &s1, n_batch, c->sm_count);
        if (!rc) rc = ensure_ws(st->ws, &s2, n_batch, c->sm_count);
        if (!rc && !st->tickets.init(c, n_batch * n_head)) rc = fail("decoder state: ticket buffer");
    }
    if (rc) {
        zwg_dec_state_destroy(st);
        return rc;
    }
    *out = st;
    return ZWG_OK;
}

int zwg_dec_state_destroy(zwg_dec_state* st) {
    if (!st) return ZWG_OK;
    int dev = -1;
    cudaGetDevice(&dev);
    cudaSetDevice(st->device);
    cudaDeviceSynchronize();
    free_all(st->self_k);
    free_all(st->self_v);
    free_all(st->cross_k);
    free_all(st->cross_v);
    st->ws.release();
    st->tickets.buf.release();
    if (dev >= 0) cudaSetDevice(dev);
    delete st;
    return ZWG_OK;
}

int zwg_dec_state_cache(const zwg_dec_state* st, size_t layer, float** self_k, float** self_v, float** cross_k,
                        float** cross_v) {
    if (!st || layer >= st->n_layer) return fail("bad state or layer");
    if (self_k) *self_k = st->self_k[layer];
    if (self_v) *self_v = st->self_v[layer];
    if (cross_k) *cross_k = st->cross_k[layer];
    if (cross_v) *cross_v = st->cross_v[layer];
    return ZWG_OK;
}

int zwg_cross_kv_set(zwg_dec_state* st, size_t layer, size_t window, const float* k, const float* v, void* stream) {
    if (!st || layer >= st->n_layer || window >= st->n_batch || !k || !v) return fail("cross_kv_set: bad arguments");
    Ctx* c = ctx_for(st->device);
    if (!c) return ZWG_ERROR;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t n = st->n_audio_ctx * st->n_state;
    cudaError_t e = cudaMemcpyAsync(st->cross_k[layer] + window * n, k, n * sizeof(float), cudaMemcpyDefault, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(st->cross_v[layer] + window * n, v, n * sizeof(float), cudaMemcpyDefault, s);
    if (e != cudaSuccess) return cuda_fail("cross_kv_set copy", e);
    return ZWG_OK;
}

int zwg_dec_step_attn(zwg_dec_state* st, size_t layer, int kind, const float* q, const float* k_new,
                      const float* v_new, size_t n_past, size_t n, float* out, void* stream) {
    if (!st || layer >= st->n_layer) return fail("dec_step_attn: bad state or layer");
    if (kind != ZWG_DEC_SELF && kind != ZWG_DEC_CROSS) return fail("dec_step_attn: unknown kind %d", kind);
    if (n == 0) return ZWG_OK;
    if (!q || !out) return fail("dec_step_attn: null q/out");
    Ctx* c = ctx_for(st->device);
    if (!c) return ZWG_ERROR;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t ns = st->n_state, nb = st->n_batch;
    zwg_attn_shape sh;
    zwg_batch b;
    const float *kp, *vp;
    if (kind == ZWG_DEC_SELF) {
        if (!k_new != !v_new) return fail("dec_step_attn: k_new and v_new must both be given or both be null");
        if (n_past + n > st->n_text_ctx) return fail("dec_step_attn: context full (%zu + %zu > %zu)", n_past, n, st->n_text_ctx);
        // the new rows land at n_past.. of every window's cache (src/decoder.zig:182-183);
        // both null: the caller's kernel has written them there already
        if (k_new) {
            const size_t row_bytes = n * ns * sizeof(float), pitch = st->n_text_ctx * ns * sizeof(float);
            cudaError_t e = cudaMemcpy2DAsync(st->self_k[layer] + n_past * ns, pitch, k_new, row_bytes, row_bytes, nb,
                                              cudaMemcpyDefault, s);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(st->self_v[layer] + n_past * ns, pitch, v_new, row_bytes, row_bytes, nb,
                                      cudaMemcpyDefault, s);
            if (e != cudaSuccess) return cuda_fail("dec_step_attn append", e);
        }
        sh = mha(n, n_past + n, ns, st->n_head, true);
        b = zwg_batch{nb, n * ns, st->n_text_ctx * ns, st->n_text_ctx * ns, n * ns};
        kp = st->self_k[layer];
        vp = st->self_v[layer];
    } else {
        sh = mha(n, st->n_audio_ctx, ns, st->n_head, false);
        b = zwg_batch{nb, n * ns, st->n_audio_ctx * ns, st->n_audio_ctx * ns, n * ns};
        kp = st->cross_k[layer];
        vp = st->cross_v[layer];
    }
    int rc = check_shape(&sh);
    if (!rc) rc = ensure_ws(st->ws, &sh, nb, c->sm_count);
    if (rc) return rc;
    int* tk = st->tickets.get(c, nb * st->n_head, s);
    if (!tk) return fail("dec_step_attn: ticket buffer");
    return run_dev(c, &sh, &b, q, kp, vp, out, st->ws.ptr, st->ws.cap, s, tk);
}

// ---- Qwen2 LLM ----------------------------------------------------------------------------

int zwg_llm_state_create(size_t n_layer, size_t n_batch, size_t n_head, size_t n_head_kv, size_t d, size_t n_ctx,
                         double rope_base, zwg_llm_state** out) {
    if (!out) return fail("null output pointer");
    *out = nullptr;
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (!n_layer || !n_batch || !n_head || !n_head_kv || n_head % n_head_kv || !d || d % 4 || !n_ctx || n_ctx % 4 ||
        !(rope_base > 0))
        return fail("llm state: bad sizes (n_head %zu, n_head_kv %zu, d %zu, n_ctx %zu)", n_head, n_head_kv, d, n_ctx);
    zwg_llm_state* st = new zwg_llm_state();
    st->device = c->device;
    st->n_layer = n_layer;
    st->n_batch = n_batch;
    st->n_head = n_head;
    st->n_head_kv = n_head_kv;
    st->d = d;
    st->n_ctx = n_ctx;
    const size_t per = n_batch * n_head_kv * d * n_ctx;
    // cache_kt is zeroed so columns beyond n_kv are finite, as the reference does (src/llm.zig:125)
    int rc = alloc_layers(st->cache_kt, n_layer, per, true);
    if (!rc) rc = alloc_layers(st->cache_v, n_layer, per, false);
    if (!rc) {
        // rotary tables in f64, cast to f32 (src/llm.zig:128-137)
        const size_t half = d / 2;
        std::vector<float> cs(n_ctx * half), sn(n_ctx * half);
        for (size_t p = 0; p < n_ctx; p++)
            for (size_t i = 0; i < half; i++) {
                const double inv = 1.0 / std::pow(rope_base, (double)(2 * i) / (double)d);
                const double ang = (double)p * inv;
                cs[p * half + i] = (float)std::cos(ang);
                sn[p * half + i] = (float)std::sin(ang);
            }
        cudaError_t e = cudaMalloc(&st->cos_tab, cs.size() * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&st->sin_tab, sn.size() * sizeof(float));
        if (e == cudaSuccess) e = cudaMemcpy(st->cos_tab, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(st->sin_tab, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) rc = cuda_fail("rope tables", e);
    }
    if (!rc) {
        // worst case of a decode step: one query over the whole context
        zwg_attn_shape s1{1, n_ctx, n_head, n_head_kv, d, n_head * d, n_head_kv * d, n_head * d, 1, n_ctx};
        rc = ensure_ws(st->ws, &s1, n_batch, c->sm_count);
        if (!rc && !st->tickets.init(c, n_batch * n_head_kv)) rc = fail("llm state: ticket buffer");
    }
    if (rc) {
        zwg_llm_state_destroy(st);
        return rc;
    }
    *out = st;
    return ZWG_OK;
}

int zwg_llm_state_destroy(zwg_llm_state* st) {
    if (!st) return ZWG_OK;
    int dev = -1;
    cudaGetDevice(&dev);
    cudaSetDevice(st->device);
    cudaDeviceSynchronize();
    free_all(st->cache_kt);
    free_all(st->cache_v);
    if (st->cos_tab) cudaFree(st->cos_tab);
    if (st->sin_tab) cudaFree(st->sin_tab);
    st->ws.release();
    st->tickets.buf.release();
    if (dev >= 0) cudaSetDevice(dev);
    delete st;
    return ZWG_OK;
}

int zwg_llm_state_cache(const zwg_llm_state* st, size_t layer, float** cache_kt, float** cache_v) {
    if (!st || layer >= st->n_layer) return fail("bad state or layer");
    if (cache_kt) *cache_kt = st->cache_kt[layer];
    if (cache_v) *cache_v = st->cache_v[layer];
    return ZWG_OK;
}

int zwg_llm_append_rope(zwg_llm_state* st, size_t layer, float* q, const float* k, const float* v, size_t n_past,
                        size_t n, void* stream) {
    if (!st || layer >= st->n_layer) return fail("llm_append_rope: bad state or layer");
    if (n == 0) return ZWG_OK;
    if (!q || !k || !v) return fail("llm_append_rope: null q/k/v");
    if (n_past + n > st->n_ctx) return fail("llm_append_rope: context full (%zu + %zu > %zu)", n_past, n, st->n_ctx);
    Ctx* c = ctx_for(st->device);
    if (!c) return ZWG_ERROR;
    const size_t kvw = st->n_head_kv * st->d;
    zwg::RopeParams p{q, k, v, st->cache_kt[layer], st->cache_v[layer], st->cos_tab, st->sin_tab, n, n_past,
                      st->n_head, st->n_head_kv, st->d, st->n_ctx, n * st->n_head * st->d, n * kvw, kvw * st->n_ctx};
    if (zwg::rope_kt_append_launch(p, st->n_batch, (cudaStream_t)stream)) return cuda_fail("rope launch", cudaGetLastError());
    return ZWG_OK;
}


int zwg_llm_attn_prefill(zwg_llm_state* st, size_t layer, const float* q, size_t n_past, size_t n, float* out,
                         void* stream) {
    return llm_attn(st, layer, q, n_past, n, out, stream);
}

int zwg_llm_attn_decode(zwg_llm_state* st, size_t layer, const float* q, size_t n_past, float* out, void* stream) {
    return llm_attn(st, layer, q, n_past, 1, out, stream);
}

}  // extern "C"
