// Internals of the C-ABI layer shared by its source files (api.cu: contexts and the
// attention entry points; state.cu: the library-owned decoder and LLM states; llm_api.cu:
// the Qwen2 decode step around the attention; dec_api.cu: the Whisper decoder step).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <algorithm>
#include <atomic>
#include <vector>

#include "../../include/zwgpu.h"

namespace zwg {
namespace capi {

struct DevBuf {
    void* ptr = nullptr;
    size_t cap = 0;
    bool ensure(size_t bytes) {
        if (bytes <= cap) return true;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
        size_t want = std::max(bytes, (size_t)256);
        if (cudaMalloc(&ptr, want) != cudaSuccess) return false;
        cap = want;
        return true;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
    }
};

struct Ctx {
    int device = -1;
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    // host-pointer calls run as a three-stage pipeline over a ring of staging slots: copies
    // in on `side`, the kernels on `stream`, copies out on `outs`, joined by events
    cudaStream_t side = nullptr;
    cudaStream_t outs = nullptr;
    static constexpr int kSlots = 3;
    cudaEvent_t ev_in[kSlots] = {}, ev_comp[kSlots] = {}, ev_free[kSlots] = {};
    int* err = nullptr;           // device error word
    // Counts the device errors sync_and_check has reported. A kernel that gave up may have
    // left a segment ticket behind, so kept-zero ticket buffers are cleared again when this
    // moved since their last clearing.
    std::atomic<unsigned> err_gen{0};
    int math = ZWG_MATH_F32;
    DevBuf q[kSlots], k[kSlots], v[kSlots], out[kSlots], ws[kSlots];
    DevBuf qh[kSlots], kh[kSlots], vh[kSlots];   // bf16 copies for the tensor-core path
};

// Segment tickets of the split decode kernels, kept by a state for its own calls (which run
// in one stream order): zero after every completed call, since the merging CTA resets its
// ticket, so a call clears them only when a device error was reported since the last
// clearing. Allocated and cleared when the state is made, so no call allocates (graph
// capture stays legal); a clearing issued while the stream is being captured runs only when
// the graph does, so it leaves the buffer marked for clearing by the next eager call.
struct Tickets {
    DevBuf buf;
    unsigned gen = 0;  // Ctx::err_gen at the last clearing
    bool init(const Ctx* c, size_t n) {
        if (!buf.ensure(std::max<size_t>(n, 1) * sizeof(int))) return false;
        if (cudaMemset(buf.ptr, 0, buf.cap) != cudaSuccess) return false;
        gen = c->err_gen.load(std::memory_order_relaxed);
        return true;
    }
    // n tickets, zero in `st`'s order, or nullptr (more than init made, or clearing failed).
    int* get(const Ctx* c, size_t n, cudaStream_t st) {
        if (!buf.ptr || n * sizeof(int) > buf.cap) return nullptr;
        const unsigned now = c->err_gen.load(std::memory_order_relaxed);
        if (gen != now) {
            cudaStreamCaptureStatus cs = cudaStreamCaptureStatusActive;
            const bool eager = cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone;
            if (cudaMemsetAsync(buf.ptr, 0, buf.cap, st) != cudaSuccess) return nullptr;
            if (eager) gen = now;
        }
        return static_cast<int*>(buf.ptr);
    }
};

// The calling thread's context (zwg_init), or nullptr with the last error set.
Ctx* cur();
// The device error word of the calling thread's context when that context is on the current
// device, else nullptr (no error is recorded either way). For launchers below the C API
// that have no context argument.
int* current_err_word();
// Record the calling thread's last error (printf format); return ZWG_ERROR.
int fail(const char* fmt, ...);
int cuda_fail(const char* what, cudaError_t e);
// Argument checks of an attention call (the reference's asserts, src/ops.zig:564-568).
int check_shape(const zwg_attn_shape* sh);
// Workspace bytes run_dev needs for this shape and batch.
size_t workspace_bytes(const zwg_attn_shape* sh, size_t n_batch, int sm_count);
// One batched attention call on device pointers (the body of zwg_attention_dev).
// tickets: n_batch * n_head_kv kept-zero ints (a state's Tickets), or nullptr to clear the
// workspace's own before a split decode kernel.
int run_dev(Ctx* c, const zwg_attn_shape* sh, const zwg_batch* b, const float* q, const float* k,
            const float* v, float* out, void* ws, size_t ws_bytes, cudaStream_t st, int* tickets = nullptr);

// The calling thread's context, which must be on `device` (the device a state lives on);
// nullptr with the last error set otherwise.
Ctx* ctx_for(int device);

}  // namespace capi
}  // namespace zwg

// Whisper decoder state (state.cu): per layer the self K/V cache and the cross K/V of
// n_batch windows, on one device.
struct zwg_dec_state {
    int device = -1;
    size_t n_layer = 0, n_batch = 0, n_state = 0, n_head = 0, n_text_ctx = 0, n_audio_ctx = 0;
    // per layer: self K/V [n_batch][n_text_ctx][n_state], cross K/V [n_batch][n_audio_ctx][n_state]
    std::vector<float*> self_k, self_v, cross_k, cross_v;
    zwg::capi::DevBuf ws;
    zwg::capi::Tickets tickets;
};

// Qwen2 LLM state (state.cu): the caches of every layer for n_batch sequences and the RoPE
// tables, on one device.
struct zwg_llm_state {
    int device = -1;
    size_t n_layer = 0, n_batch = 0, n_head = 0, n_head_kv = 0, d = 0, n_ctx = 0;
    // per layer: cache_kt [n_batch][n_head_kv][d][n_ctx] (zeroed), cache_v [n_batch][n_ctx][n_head_kv*d]
    std::vector<float*> cache_kt, cache_v;
    float* cos_tab = nullptr;  // [n_ctx][d/2]
    float* sin_tab = nullptr;
    zwg::capi::DevBuf ws;
    zwg::capi::Tickets tickets;
};

namespace zwg {
namespace capi {
// Causal GQA attention of q [n_batch][n][n_head*d] over one layer's caches, n_kv = n_past + n
// (the body of zwg_llm_attn_prefill / _decode).
int llm_attn(zwg_llm_state* st, size_t layer, const float* q, size_t n_past, size_t n, float* out, void* stream);
}  // namespace capi
}  // namespace zwg
