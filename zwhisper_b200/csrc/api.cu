// C-ABI layer of libzwgpu (declared in include/zwgpu.h): per-device contexts, argument
// checks mirroring the reference's asserts (src/ops.zig:564-568), host-pointer drop-in
// entry points and device-pointer batched entry points.
#include "../../include/zwgpu.h"
#include "common.cuh"
#include "kernels.h"
#include "api_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>
#include <string>

namespace zwg {
namespace capi {

std::mutex g_mu;
Ctx* g_ctx[64] = {};
thread_local Ctx* t_cur = nullptr;
thread_local std::string t_err;

int fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    return ZWG_ERROR;
}

int cuda_fail(const char* what, cudaError_t e) {
    return fail("%s: %s", what, cudaGetErrorString(e));
}

Ctx* cur() {
    if (!t_cur) fail("zwg_init was not called on this thread");
    return t_cur;
}

int* current_err_word() {
    int dev = -1;
    if (!t_cur || cudaGetDevice(&dev) != cudaSuccess || dev != t_cur->device) return nullptr;
    return t_cur->err;
}

// Elements spanned by `rows` rows of `width` elements at `stride`.
size_t span(size_t rows, size_t stride, size_t width) { return rows ? (rows - 1) * stride + width : 0; }

int check_shape(const zwg_attn_shape* sh) {
    if (!sh) return fail("null shape");
    if (sh->n_head == 0 || sh->n_head_kv == 0 || sh->n_head % sh->n_head_kv)
        return fail("n_head (%zu) must be a positive multiple of n_head_kv (%zu)", sh->n_head, sh->n_head_kv);
    if (sh->d == 0 || sh->d % 4 || sh->d > 256) return fail("d = %zu: need a multiple of 4 up to 256", sh->d);
    if (sh->q_stride < sh->n_head * sh->d || sh->out_stride < sh->n_head * sh->d)
        return fail("q/out stride smaller than n_head * d");
    if (sh->kv_stride < sh->n_head_kv * sh->d) return fail("kv stride smaller than n_head_kv * d");
    if (sh->causal && sh->n_kv < sh->n_q) return fail("causal attention needs n_kv >= n_q (%zu < %zu)", sh->n_kv, sh->n_q);
    if (sh->kt_stride && sh->kt_stride < sh->n_kv) return fail("kt_stride %zu < n_kv %zu", sh->kt_stride, sh->n_kv);
    if (sh->kt_stride % 4) return fail("kt_stride must be a multiple of 4");
    if (sh->n_kv > (1u << 30) || sh->n_q > (1u << 30)) return fail("sequence too long");
    return ZWG_OK;
}

struct Extents {
    size_t q, k, v, out;
};

Extents extents(const zwg_attn_shape* sh) {
    Extents e;
    e.q = span(sh->n_q, sh->q_stride, sh->n_head * sh->d);
    e.k = sh->kt_stride ? sh->n_head_kv * sh->d * sh->kt_stride : span(sh->n_kv, sh->kv_stride, sh->n_head_kv * sh->d);
    e.v = span(sh->n_kv, sh->kv_stride, sh->n_head_kv * sh->d);
    e.out = span(sh->n_q, sh->out_stride, sh->n_head * sh->d);
    return e;
}

// Decode-shaped calls (few query rows per kv head) take the TMA decode kernel; an empty
// key range (its rows are all zeros) takes the tiled kernel, which writes them.
bool use_decode(const zwg_attn_shape* sh) {
    const size_t rows = sh->n_q * (sh->n_head / sh->n_head_kv);
    return sh->n_kv > 0 && zwg::decode_supported(sh->d, rows, sh->kt_stride);
}

struct Plan {
    bool decode;
    int n_splits, chunk;
    size_t ws_bytes;
};

Plan plan_for(const zwg_attn_shape* sh, size_t n_batch, int sm_count) {
    Plan pl{};
    pl.decode = use_decode(sh);
    if (pl.decode) {
        int grid = 1, p_max = 1;
        zwg::decode_tma_plan(n_batch, sh->n_head_kv, sh->n_kv, sm_count, &grid, &p_max);
        const size_t rows = sh->n_q * (sh->n_head / sh->n_head_kv);
        pl.ws_bytes = zwg::decode_tma_workspace_bytes(n_batch, sh->n_head_kv, rows, sh->d, p_max);
        // enough for the tensor-core decode too (tf32 math mode), whichever mode runs
        if (sh->n_q == 1 && sh->kt_stride)
            pl.ws_bytes = std::max(pl.ws_bytes, zwg::decode_tc_workspace_bytes(n_batch, sh->n_head_kv, rows, sh->d));
    }
    return pl;
}

size_t workspace_bytes(const zwg_attn_shape* sh, size_t n_batch, int sm_count) {
    return plan_for(sh, n_batch, sm_count).ws_bytes;
}

int run_dev(Ctx* c, const zwg_attn_shape* sh, const zwg_batch* b, const float* q, const float* k,
            const float* v, float* out, void* ws, size_t ws_bytes, cudaStream_t st, int* tickets) {
    const size_t nb = b ? b->n_batch : 1;
    if (nb == 0 || sh->n_q == 0) return ZWG_OK;
    const Plan pl = plan_for(sh, nb, c->sm_count);
    int rc;
    if (pl.decode) {
        if (ws_bytes < pl.ws_bytes) return fail("workspace too small: %zu < %zu bytes", ws_bytes, pl.ws_bytes);
        if (((uintptr_t)k | (uintptr_t)v | (uintptr_t)q) & 15)
            return fail("decode kernel needs 16-byte aligned q, k, v");
        if ((sh->kv_stride | sh->q_stride) % 4) return fail("decode kernel needs strides that are multiples of 4");
        zwg::DecodeParams p{};
        p.q = q; p.k = k; p.v = v; p.out = out; p.ws = (float*)ws;
        p.n_q = sh->n_q; p.n_kv = sh->n_kv; p.n_head = sh->n_head; p.n_head_kv = sh->n_head_kv; p.d = sh->d;
        p.q_stride = sh->q_stride; p.kv_stride = sh->kv_stride; p.out_stride = sh->out_stride;
        p.kt_stride = sh->kt_stride; p.causal = sh->causal ? 1 : 0;
        p.n_splits = pl.n_splits; p.chunk = pl.chunk;
        p.tickets = tickets;
        if (b) { p.q_bs = b->q_batch_stride; p.k_bs = b->k_batch_stride; p.v_bs = b->v_batch_stride; p.out_bs = b->out_batch_stride; }
        if (p.k_bs % 4 || p.v_bs % 4 || p.q_bs % 4) return fail("decode kernel needs batch strides that are multiples of 4");
        if ((c->math & ZWG_MATH_TF32) && zwg::decode_tc_supported(p, nb)) {
            rc = zwg::decode_tc_launch(p, nb, c->sm_count, c->err, st);
        } else {
            if (!zwg::decode_tma_supported(p)) return fail("decode shape not supported by the TMA decode kernel");
            rc = zwg::decode_tma_launch(p, nb, c->sm_count, c->err, st);
        }
    } else {
        zwg::FlashParams p{};
        p.q = q; p.k = k; p.v = v; p.out = out;
        p.n_q = sh->n_q; p.n_kv = sh->n_kv; p.n_head = sh->n_head; p.n_head_kv = sh->n_head_kv; p.d = sh->d;
        p.q_stride = sh->q_stride; p.kv_stride = sh->kv_stride; p.out_stride = sh->out_stride;
        p.kt_stride = sh->kt_stride; p.causal = sh->causal ? 1 : 0;
        if (b) { p.q_bs = b->q_batch_stride; p.k_bs = b->k_batch_stride; p.v_bs = b->v_batch_stride; p.out_bs = b->out_batch_stride; }
        if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 3) return fail("f32 buffers must be 4-byte aligned");
        if ((c->math & ZWG_MATH_TF32) && zwg::prefill_tc_supported(p, nb))
            rc = zwg::prefill_tc_launch(p, nb, c->sm_count, c->err, st);
        else
            rc = zwg::flash_f32_launch(p, nb, st);
    }
    if (rc) return cuda_fail("kernel launch", cudaGetLastError());
    return ZWG_OK;
}

int sync_and_check(Ctx* c, cudaStream_t st) {
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail("stream synchronize", e);
    int h = 0;
    e = cudaMemcpy(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail("error word read", e);
    if (h) {
        cudaMemset(c->err, 0, sizeof(int));
        c->err_gen.fetch_add(1, std::memory_order_relaxed);
        if (h == zwg::kErrTimeout) {
            fail("a device-side wait timed out");
            return ZWG_TIMEOUT;
        }
        return fail("device error code %d", h);
    }
    return ZWG_OK;
}

}  // namespace capi
}  // namespace zwg

using namespace zwg::capi;

namespace zwg {
int set_last_error(const char* msg) { return fail("%s", msg); }
int set_last_error_cuda(const char* what, cudaError_t e) { return cuda_fail(what, e); }
}  // namespace zwg

extern "C" {

int zwg_version(void) { return 1; }

int zwg_set_math(int mode) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (mode & ~(ZWG_MATH_BF16 | ZWG_MATH_TF32)) return fail("unknown math mode %d", mode);
    c->math = mode;
    return ZWG_OK;
}

int zwg_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int zwg_init(int device) {
    int n = zwg_device_count();
    if (device < 0 || device >= n || device >= 64) return fail("device %d not available (%d visible)", device, n);
    std::lock_guard<std::mutex> lk(g_mu);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail("cudaSetDevice", e);
    if (!g_ctx[device]) {
        Ctx* c = new Ctx();
        c->device = device;
        cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
        if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaStreamCreateWithFlags(&c->outs, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaMalloc(&c->err, sizeof(int))) != cudaSuccess ||
            (e = cudaMemset(c->err, 0, sizeof(int))) != cudaSuccess) {
            delete c;
            return cuda_fail("context set-up", e);
        }
        for (int i = 0; i < Ctx::kSlots && e == cudaSuccess; i++) {
            if ((e = cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming)) == cudaSuccess &&
                (e = cudaEventCreateWithFlags(&c->ev_comp[i], cudaEventDisableTiming)) == cudaSuccess)
                e = cudaEventCreateWithFlags(&c->ev_free[i], cudaEventDisableTiming);
        }
        if (e != cudaSuccess) {
            delete c;
            return cuda_fail("context set-up", e);
        }
        g_ctx[device] = c;
    }
    t_cur = g_ctx[device];
    return ZWG_OK;
}

int zwg_shutdown(void) {
    Ctx* c = t_cur;
    if (!c) return ZWG_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    cudaStreamSynchronize(c->side);
    cudaStreamSynchronize(c->outs);
    for (int i = 0; i < Ctx::kSlots; i++) {
        c->q[i].release(); c->k[i].release(); c->v[i].release(); c->out[i].release(); c->ws[i].release();
        c->qh[i].release(); c->kh[i].release(); c->vh[i].release();
        cudaEventDestroy(c->ev_in[i]);
        cudaEventDestroy(c->ev_comp[i]);
        cudaEventDestroy(c->ev_free[i]);
    }
    cudaFree(c->err);
    cudaStreamDestroy(c->stream);
    cudaStreamDestroy(c->side);
    cudaStreamDestroy(c->outs);
    g_ctx[c->device] = nullptr;
    delete c;
    t_cur = nullptr;
    return ZWG_OK;
}

size_t zwg_last_error(char* buf, size_t len) {
    if (buf && len) {
        size_t n = std::min(len - 1, t_err.size());
        memcpy(buf, t_err.data(), n);
        buf[n] = 0;
    }
    return t_err.size();
}

int zwg_sync(void) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail("device synchronize", e);
    return sync_and_check(c, c->stream);
}

size_t zwg_attention_workspace(const zwg_attn_shape* sh, const zwg_batch* b) {
    if (check_shape(sh) != ZWG_OK) return 0;
    int sms = 148;
    if (t_cur) sms = t_cur->sm_count;
    return plan_for(sh, b ? b->n_batch : 1, sms).ws_bytes;
}

int zwg_attention_dev(const zwg_attn_shape* sh, const zwg_batch* b, const float* q, const float* k,
                      const float* v, float* out, void* workspace, size_t workspace_bytes, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    int rc = check_shape(sh);
    if (rc) return rc;
    if (sh->n_q && (!q || !out)) return fail("null q/out");
    if (sh->n_kv && (!k || !v)) return fail("null k/v");
    cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
    return run_dev(c, sh, b, q, k, v, out, workspace, workspace_bytes, st);
}

// An encoder-shaped call the tcgen05 kernel computes exactly as specified.
static bool tc_eligible(const zwg_attn_shape* sh) {
    const size_t ns = sh->n_head * 64;
    return sh->d == 64 && !sh->causal && sh->n_head == sh->n_head_kv && sh->kt_stride == 0 &&
           sh->n_q == sh->n_kv && sh->n_q > 0 && sh->q_stride == ns && sh->kv_stride == ns &&
           sh->out_stride == ns && sh->n_head <= 64 && sh->n_q <= (1u << 20);
}

// Host-pointer path: stage inputs, run, copy the written head columns back. The batch runs in
// chunks through a ring of device staging slots as a three-stage pipeline: copies in on one
// stream, the kernels on another, copies out on a third, so the host-to-device link (the
// larger direction for attention: q, k and v in, one output back) stays busy while earlier
// chunks compute and return. A slot is refilled only after its previous chunk's copy out.
static int host_call(Ctx* c, const zwg_attn_shape* sh, const zwg_batch* b, const float* q, const float* k,
                     const float* v, float* out) {
    const Extents ex = extents(sh);
    const size_t nb = b ? b->n_batch : 1;
    if (nb == 0 || sh->n_q == 0) return ZWG_OK;
    const size_t qbs = b ? b->q_batch_stride : 0, kbs = b ? b->k_batch_stride : 0;
    const size_t vbs = b ? b->v_batch_stride : 0, obs = b ? b->out_batch_stride : 0;
    // items per chunk: at most 256 MB of f32 staging per slot, and about twelve chunks when
    // the batch allows. The first chunks grow 1, 2, 4, ... up to that size and the last ones
    // shrink the same way: the copies in of the first chunk run with nothing beside them and
    // the kernels and copies out of the last one likewise, so each call's fill and drain move
    // one item, not a full chunk (12 calls of 64 windows: 2 ms per call before).
    const size_t item_bytes = (ex.q + ex.k + ex.v + ex.out) * sizeof(float);
    size_t per = std::max<size_t>(1, (size_t)(256u << 20) / std::max<size_t>(item_bytes, 1));
    per = std::min(per, std::max<size_t>(1, (nb + 11) / 12));
    std::vector<size_t> ramp;  // 1, 2, 4, ... below per, while both ramps fit in the batch
    {
        size_t sum = 0;
        for (size_t r = 1; r < per && 2 * (sum + r) <= nb; r *= 2) {
            ramp.push_back(r);
            sum += r;
        }
    }
    size_t ramp_sum = 0;
    for (size_t r : ramp) ramp_sum += r;
    auto chunk_items = [&](size_t chunk, size_t i0) -> size_t {
        if (chunk < ramp.size()) return ramp[chunk];
        const size_t left = nb - i0;
        if (left <= ramp_sum) {
            // the falling ramp: the largest power of two of the rising one that leaves the
            // rest to smaller chunks
            for (size_t k = ramp.size(); k-- > 0;)
                if (ramp[k] <= left) return ramp[k];
            return left;
        }
        return std::min(per, left - ramp_sum);
    };
    const zwg_attn_shape& s = *sh;
    const bool tc = (c->math & ZWG_MATH_BF16) && tc_eligible(sh);
    const size_t dq = ex.q, dk = ex.k, dv = ex.v, dout = ex.out;
    cudaError_t e = cudaSuccess;
    int rc = ZWG_OK;
    size_t chunk = 0;
    for (size_t i0 = 0, n = 0; i0 < nb && rc == ZWG_OK; i0 += n, chunk++) {
        n = std::min(chunk_items(chunk, i0), nb - i0);
        const int slot = (int)(chunk % Ctx::kSlots);
        zwg_batch db{n, dq, dk, dv, dout};
        Plan pl = plan_for(sh, n, c->sm_count);
        // the slot's previous chunk has left the device before its buffers are reused (the
        // host waits here so that a buffer can grow safely)
        if (chunk >= (size_t)Ctx::kSlots && (e = cudaEventSynchronize(c->ev_free[slot])) != cudaSuccess) {
            rc = cuda_fail("staging slot wait", e);
            break;
        }
        if (!c->q[slot].ensure(per * dq * 4 + 16) || !c->k[slot].ensure(per * dk * 4 + 16) ||
            !c->v[slot].ensure(per * dv * 4 + 16) || !c->out[slot].ensure(per * dout * 4 + 16) ||
            !c->ws[slot].ensure(pl.ws_bytes + 16) ||
            (tc && (!c->qh[slot].ensure(per * dq * 2 + 16) || !c->kh[slot].ensure(per * dq * 2 + 16) ||
                    !c->vh[slot].ensure(per * dq * 2 + 16)))) {
            rc = fail("device staging allocation failed");
            break;
        }
        // ---- copies in: one copy per tensor when the chunk's items lie back to back on the
        // host (batch stride = extent), else one per item (each copy has a fixed cost)
        auto copy_in = [&](float* dst, const float* src, size_t d, size_t bs) -> cudaError_t {
            if (!d) return cudaSuccess;
            if (bs == d || n == 1)
                return cudaMemcpyAsync(dst, src + i0 * bs, n * d * 4, cudaMemcpyHostToDevice, c->side);
            cudaError_t r = cudaSuccess;
            for (size_t j = 0; j < n && r == cudaSuccess; j++)
                r = cudaMemcpyAsync(dst + j * d, src + (i0 + j) * bs, d * 4, cudaMemcpyHostToDevice, c->side);
            return r;
        };
        e = copy_in((float*)c->q[slot].ptr, q, dq, qbs);
        if (e == cudaSuccess) e = copy_in((float*)c->k[slot].ptr, k, dk, kbs);
        if (e == cudaSuccess) e = copy_in((float*)c->v[slot].ptr, v, dv, vbs);
        if (e == cudaSuccess) e = cudaEventRecord(c->ev_in[slot], c->side);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->stream, c->ev_in[slot], 0);
        if (e != cudaSuccess) {
            rc = cuda_fail("host to device copy", e);
            break;
        }
        // ---- the kernels
        cudaStream_t st = c->stream;
        if (tc) {
            const size_t ne = n * dq;  // q, k, v have the same extent here
            if (zwg::f32_to_bf16_launch((float*)c->q[slot].ptr, (uint16_t*)c->qh[slot].ptr, ne, st) ||
                zwg::f32_to_bf16_launch((float*)c->k[slot].ptr, (uint16_t*)c->kh[slot].ptr, ne, st) ||
                zwg::f32_to_bf16_launch((float*)c->v[slot].ptr, (uint16_t*)c->vh[slot].ptr, ne, st)) {
                rc = cuda_fail("bf16 conversion", cudaGetLastError());
                break;
            }
            zwg::EncTcParams tp{(uint16_t*)c->qh[slot].ptr, (uint16_t*)c->kh[slot].ptr, (uint16_t*)c->vh[slot].ptr,
                                (float*)c->out[slot].ptr, (int)n, (int)s.n_q, (int)s.n_head, c->err};
            rc = zwg::enc_tc_launch(tp, st) ? cuda_fail("enc_attn launch", cudaGetLastError()) : ZWG_OK;
        } else {
            rc = run_dev(c, &s, &db, (float*)c->q[slot].ptr, (float*)c->k[slot].ptr, (float*)c->v[slot].ptr,
                         (float*)c->out[slot].ptr, c->ws[slot].ptr, c->ws[slot].cap, st);
        }
        if (rc) break;
        if ((e = cudaEventRecord(c->ev_comp[slot], st)) == cudaSuccess)
            e = cudaStreamWaitEvent(c->outs, c->ev_comp[slot], 0);
        // ---- copies out: only the head columns of each output row are written, as in the
        // reference; rows without gaps and items back to back on the host go in one copy
        if (e == cudaSuccess && s.out_stride == s.n_head * s.d && (obs == dout || n == 1)) {
            e = cudaMemcpyAsync(out + i0 * obs, c->out[slot].ptr, n * dout * 4, cudaMemcpyDeviceToHost, c->outs);
        } else {
            for (size_t j = 0; j < n && e == cudaSuccess; j++)
                e = cudaMemcpy2DAsync(out + (i0 + j) * obs, s.out_stride * 4, (float*)c->out[slot].ptr + j * dout,
                                      s.out_stride * 4, s.n_head * s.d * 4, s.n_q, cudaMemcpyDeviceToHost, c->outs);
        }
        if (e == cudaSuccess) e = cudaEventRecord(c->ev_free[slot], c->outs);
        if (e != cudaSuccess) rc = cuda_fail("device to host copy", e);
    }
    // every stage drains before the call returns, also after an error
    const int r1 = sync_and_check(c, c->side);
    const int r2 = sync_and_check(c, c->stream);
    const int r3 = sync_and_check(c, c->outs);
    return rc ? rc : r1 ? r1 : r2 ? r2 : r3;
}

int zwg_attention(const zwg_attn_shape* sh, const float* q, const float* k, const float* v, float* out) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    int rc = check_shape(sh);
    if (rc) return rc;
    if (sh->n_q && (!q || !out)) return fail("null q/out");
    if (sh->n_kv && (!k || !v)) return fail("null k/v");
    return host_call(c, sh, nullptr, q, k, v, out);
}

int zwg_attention_mha(const float* q, const float* k, const float* v, size_t n_q, size_t n_kv, size_t n_state,
                      size_t n_head, int32_t causal, float* out) {
    if (n_head == 0 || n_state % n_head) return fail("n_state %zu not divisible by n_head %zu", n_state, n_head);
    zwg_attn_shape sh{n_q, n_kv, n_head, n_head, n_state / n_head, n_state, n_state, n_state, causal, 0};
    return zwg_attention(&sh, q, k, v, out);
}

int zwg_attention_batch_host(const zwg_attn_shape* sh, const zwg_batch* b, const float* q, const float* k,
                             const float* v, float* out) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    int rc = check_shape(sh);
    if (rc) return rc;
    if (!b) return fail("null batch");
    return host_call(c, sh, b, q, k, v, out);
}

int zwg_f32_to_bf16(const float* x, uint16_t* y, size_t n, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
    if (zwg::f32_to_bf16_launch(x, y, n, st)) return fail("f32_to_bf16: unaligned buffers or launch failure");
    return ZWG_OK;
}

int zwg_enc_attn_bf16(size_t n_batch, size_t n_ctx, size_t n_head, const uint16_t* q, const uint16_t* k,
                      const uint16_t* v, float* out, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (n_batch == 0 || n_ctx == 0) return ZWG_OK;
    if (n_head == 0 || n_head > 64 || n_ctx > (1u << 20) || n_batch > 65535) return fail("enc_attn: bad sizes");
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15) return fail("enc_attn: q/k/v must be 16-byte aligned");
    if (((uintptr_t)out) & 15) return fail("enc_attn: out must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
    zwg::EncTcParams p{q, k, v, out, (int)n_batch, (int)n_ctx, (int)n_head, c->err};
    if (zwg::enc_tc_launch(p, st)) return cuda_fail("enc_attn launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_selftest_timeout(void) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    int* gave_up = nullptr;
    cudaError_t e = cudaMalloc(&gave_up, sizeof(int));
    if (e != cudaSuccess) return cuda_fail("selftest allocation", e);
    int h = 0;
    if ((e = cudaMemsetAsync(gave_up, 0, sizeof(int), c->stream)) != cudaSuccess) {
        cudaFree(gave_up);
        return cuda_fail("selftest", e);
    }
    if (zwg::wait_timeout_selftest_launch(c->err, gave_up, c->stream)) {
        cudaFree(gave_up);
        return cuda_fail("selftest launch", cudaGetLastError());
    }
    const int rc = sync_and_check(c, c->stream);  // expected: ZWG_TIMEOUT, error word cleared
    e = cudaMemcpy(&h, gave_up, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(gave_up);
    if (e != cudaSuccess) return cuda_fail("selftest readback", e);
    if (rc == ZWG_TIMEOUT && h == 1) return ZWG_TIMEOUT;
    return fail("selftest: the bounded wait did not report a timeout (rc %d, gave_up %d)", rc, h);
}

int zwg_q8_quantize(const float* w, size_t n, size_t k, int8_t* q, float* scales, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (k == 0 || k % 32) return fail("q8_quantize: k = %zu must be a positive multiple of 32", k);
    if (n && (!w || !q || !scales)) return fail("q8_quantize: null buffer");
    if (n * (k / 32) > (1ull << 40)) return fail("q8_quantize: matrix too large");
    if (zwg::q8_quantize_launch(w, n, k, q, scales, (cudaStream_t)stream)) return cuda_fail("q8_quantize launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_linear_q8(const float* x, size_t m, size_t k, const int8_t* q, const float* scales, const float* bias,
                  size_t n, float* out, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (k == 0 || k % 32) return fail("linear_q8: k = %zu must be a positive multiple of 32", k);
    if (m == 0 || n == 0) return ZWG_OK;
    if (!x || !q || !scales || !out) return fail("linear_q8: null buffer");
    if (((uintptr_t)x | (uintptr_t)q) & 15) return fail("linear_q8: x and q must be 16-byte aligned");
    if (((uintptr_t)scales | (uintptr_t)out | (uintptr_t)bias) & 3) return fail("linear_q8: f32 buffers must be 4-byte aligned");
    if (n >= (1u << 30) || k >= (1u << 30)) return fail("linear_q8: matrix too large");
    if (zwg::q8_linear_launch(x, m, k, q, scales, bias, n, zwg::LIN_STORE, out, (cudaStream_t)stream))
        return cuda_fail("linear_q8 launch", cudaGetLastError());
    return ZWG_OK;
}

int zwg_rope_kt_append(size_t n_batch, size_t n, size_t n_past, size_t n_head, size_t n_head_kv, size_t d,
                       size_t n_ctx, float* q, const float* k, const float* v, float* cache_kt, float* cache_v,
                       const float* cos_tab, const float* sin_tab, size_t q_bstride, size_t kv_bstride,
                       size_t cache_bstride, void* stream) {
    Ctx* c = cur();
    if (!c) return ZWG_ERROR;
    if (d == 0 || d % 2) return fail("rope: d must be even");
    if (n_past + n > n_ctx) return fail("rope: context full (%zu + %zu > %zu)", n_past, n, n_ctx);
    if (n_head_kv == 0 || n_head % n_head_kv) return fail("rope: bad head counts");
    cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
    zwg::RopeParams p{q, k, v, cache_kt, cache_v, cos_tab, sin_tab, n, n_past, n_head, n_head_kv, d, n_ctx,
                      q_bstride, kv_bstride, cache_bstride};
    if (zwg::rope_kt_append_launch(p, n_batch, st)) return cuda_fail("rope launch", cudaGetLastError());
    return ZWG_OK;
}

}  // extern "C"
