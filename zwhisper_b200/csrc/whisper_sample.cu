// Whisper's greedy long-form decoding rules on the device (row f2 of the path: the host
// sampling rules of the transcription driver, so a window's tokens stay on the GPU).
//
// whisper_sample_kernel / whisper_step_kernel restate Engine.sample
// (src/transcribe.zig:491-580) for one window per block of 1024 threads:
//   1. suppression: eot and " " on the first token, the special tokens always, timestamp
//      pairing (after two timestamps no timestamp, after text + timestamp no text), the
//      initial-timestamp bound and the no-going-back bound of the window;
//   2. the hotword bias (applyHotwords, src/transcribe.zig:176-193), by one thread in the
//      forms' order so repeated additions to one logit round as the reference's do;
//   3. log-probabilities: lse = log(sum exp(l - max)) + max over the finite logits, then the
//      timestamp block's log-sum-exp of (l - lse) against the best text log-probability; a
//      winning block suppresses every text token;
//   4. the argmax (first index of the largest logit; 0 when none is finite) and the best
//      timestamp (first index of the largest logit from `beg` on; `beg` when none).
// The logits row is modified in place as the reference modifies Engine.logits. The sums of
// step 3 run in another order than the reference's vector loop and use CUDA's expf/logf, so
// they agree to f32 rounding; every other step is exact.
//
// whisper_step_kernel also does the loop body's bookkeeping (src/transcribe.zig:319-364):
// the token and the best timestamp are appended to the window's arrays on the device, and
// seek_delta, has_ts, result_len, failed and done are updated; a done window is skipped.
// zwg_whisper_decode_q8 drives the whole window loop: Decoder.forward of the prompt, then
// step and forward in turn, the host reading only the windows' done flags every few steps.
#include <cuda_runtime.h>

#include <vector>

#include "../../include/zwgpu.h"
#include "api_internal.h"
#include "common.cuh"
#include "kernels.h"

using namespace zwg::capi;

namespace zwg {
namespace ws {

constexpr int THREADS = 1024;
constexpr int WARPS = THREADS / 32;

// The rules with the derived limit of the first timestamp, passed by value to the kernels.
struct Rules {
    int eot, sot, translate, transcribe, solm, prev, nosp, not_, beg, space;
    int n_audio_ctx;
    int tid0_initial;          // round(max_initial_ts / (30 / n_audio_ctx)); < 0: rule off
    float hotword_bias;
    const int32_t* hot_tokens;
    const int32_t* hot_offsets;
    int n_hot;
};

struct ArgMax {
    float v;
    int i;
};

// larger value wins; equal values: the smaller index (the first, as the reference's scan)
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < WARPS ? red[l] : -INFINITY;
    return warp_max(v);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < WARPS ? red[l] : 0.f;
    return warp_sum(v);
}

__device__ __forceinline__ ArgMax warp_argmax(ArgMax a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
        a = better(a, b);
    }
    return a;
}

__device__ __forceinline__ ArgMax block_argmax(ArgMax a, float* redv, int* redi) {
    a = warp_argmax(a);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) {
        redv[w] = a.v;
        redi[w] = a.i;
    }
    __syncthreads();
    ArgMax b{-INFINITY, 0x7fffffff};
    if (l < WARPS) b = ArgMax{redv[l], redi[l]};
    return warp_argmax(b);
}

// Engine.sample on one logits row with all THREADS threads of the block; returns (id, tid)
// in every thread.
__device__ void sample_row(float* lg, int n, const int32_t* cur, int n_cur, bool is_initial, bool has_ts,
                           int seek_delta, const Rules& R, int* out_id, int* out_tid) {
    __shared__ float redv[WARPS];
    __shared__ int redi[WARPS];
    const int beg = R.beg;
    // 1. suppression (src/transcribe.zig:498-530)
    const bool last_ts = n_cur > 0 && cur[n_cur - 1] >= beg;
    const bool pen_ts = n_cur < 2 || cur[n_cur - 2] >= beg;
    const int init_cut = (is_initial && R.tid0_initial >= 0 && beg + R.tid0_initial + 1 < n) ? beg + R.tid0_initial + 1
                                                                                              : 0x7fffffff;
    const int back_end = has_ts ? beg + seek_delta / 2 : beg;  // timestamps [beg, back_end) off
    for (int i = threadIdx.x; i < n; i += THREADS) {
        bool off = i == R.not_ || i == R.sot || i == R.nosp || i == R.solm || i == R.translate ||
                   i == R.transcribe || i == R.prev;
        off |= is_initial && (i == R.eot || i == R.space);
        if (last_ts) off |= pen_ts ? i >= beg : i < R.eot;
        off |= i >= init_cut;
        off |= i >= beg && i < back_end;
        if (off) lg[i] = -INFINITY;
    }
    __syncthreads();
    // 2. hotwords (src/transcribe.zig:176-193): one thread, the forms in order
    if (threadIdx.x == 0 && R.n_hot > 0) {
        for (int f = 0; f < R.n_hot; f++) {
            const int32_t* form = R.hot_tokens + R.hot_offsets[f];
            const int len = R.hot_offsets[f + 1] - R.hot_offsets[f];
            if (len <= 0) continue;
            int p = min(len - 1, n_cur);
            for (; p > 0; p--) {
                bool eq = true;
                for (int u = 0; u < p && eq; u++) eq = form[u] == cur[n_cur - p + u];
                if (eq) break;
            }
            const int next = form[p];
            if (next >= 0 && next < R.eot && next < n) lg[next] = lg[next] + (p == 0 ? R.hotword_bias * 0.5f : R.hotword_bias);
        }
    }
    __syncthreads();
    // 3. log-probabilities and the timestamp block against the best text token
    float mx = -INFINITY, mx_text = -INFINITY, mx_ts = -INFINITY;
    for (int i = threadIdx.x; i < n; i += THREADS) {
        const float v = lg[i];
        mx = fmaxf(mx, v);
        if (i < beg) mx_text = fmaxf(mx_text, v);
        else mx_ts = fmaxf(mx_ts, v);
    }
    mx = block_max(mx, redv);
    mx_text = block_max(mx_text, redv);
    mx_ts = block_max(mx_ts, redv);
    float s = 0.f;
    if (mx > -INFINITY)
        for (int i = threadIdx.x; i < n; i += THREADS) {
            const float v = lg[i];
            if (v > -INFINITY) s += expf(v - mx);
        }
    s = block_sum(s, redv);
    const float lse = logf(s) + mx;
    // max over the block of (l - lse) is (max l) - lse: rounding is monotonic
    const float text_max = mx_text > -INFINITY ? mx_text - lse : -INFINITY;
    const float ts_max = mx_ts > -INFINITY ? mx_ts - lse : -INFINITY;
    float ts_lp = -INFINITY;
    if (ts_max > -INFINITY) {
        float acc = 0.f;
        for (int i = beg + threadIdx.x; i < n; i += THREADS) {
            const float v = lg[i];
            if (v > -INFINITY) acc += expf((v - lse) - ts_max);
        }
        acc = block_sum(acc, redv);
        ts_lp = logf(acc) + ts_max;
    }
    const bool text_off = ts_lp > text_max;
    // 4. argmax and the best timestamp (src/transcribe.zig:563-579)
    ArgMax best{-INFINITY, 0}, tbest{-INFINITY, beg};
    for (int i = threadIdx.x; i < n; i += THREADS) {
        float v = lg[i];
        if (i < beg && text_off) {
            lg[i] = -INFINITY;
            v = -INFINITY;
        }
        if (v > -INFINITY) {
            best = better(best, ArgMax{v, i});
            if (i >= beg) tbest = better(tbest, ArgMax{v, i});
        }
    }
    best = block_argmax(best, redv, redi);
    tbest = block_argmax(tbest, redv, redi);
    *out_id = best.v > -INFINITY ? best.i : 0;
    *out_tid = tbest.v > -INFINITY ? tbest.i : beg;
}

// zwg_whisper_sample: one block per row b.
__global__ void __launch_bounds__(THREADS) whisper_sample_kernel(float* logits, int n_vocab, const int32_t* tokens,
                                                                 size_t tokens_stride, const int32_t* n_tokens,
                                                                 const int32_t* has_ts, const int32_t* seek_delta,
                                                                 Rules R, int32_t* out_id, int32_t* out_tid) {
    const size_t b = blockIdx.x;
    const int n_cur = n_tokens ? n_tokens[b] : 0;
    const int32_t* cur = tokens ? tokens + b * tokens_stride : nullptr;
    const bool hts = has_ts ? has_ts[b] != 0 : false;
    const int sd = seek_delta ? seek_delta[b] : 2 * R.n_audio_ctx;
    int id, tid;
    sample_row(logits + b * (size_t)n_vocab, n_vocab, cur, n_cur, n_cur == 0, hts, sd, R, &id, &tid);
    if (threadIdx.x == 0) {
        out_id[b] = id;
        out_tid[b] = tid;
    }
}

__global__ void whisper_window_init_kernel(zwg_whisper_window* win, int n, int n_audio_ctx) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    zwg_whisper_window w = win[b];
    w.n_tokens = 0;
    w.seek_delta = 2 * n_audio_ctx;
    w.has_ts = 0;
    w.result_len = 0;
    w.failed = 0;
    w.done = 0;
    win[b] = w;
}

// zwg_whisper_step: sample, then the loop body's bookkeeping (src/transcribe.zig:319-364).
__global__ void __launch_bounds__(THREADS) whisper_step_kernel(float* logits, int n_vocab, zwg_whisper_window* win,
                                                               int32_t* tokens, int32_t* tids, size_t cap, Rules R,
                                                               int n_max, int32_t* next_token) {
    const size_t b = blockIdx.x;
    __shared__ zwg_whisper_window w;
    if (threadIdx.x == 0) w = win[b];
    __syncthreads();
    if (w.done || w.n_tokens >= n_max || (size_t)w.n_tokens >= cap) {
        // the window has ended: nothing is sampled; the decoder keeps a valid input token
        if (threadIdx.x == 0) {
            next_token[b] = w.n_tokens > 0 ? tokens[b * cap + w.n_tokens - 1] : R.eot;
            if (!w.done) {
                win[b].done = 1;
            }
        }
        return;
    }
    const int i = w.n_tokens;
    int32_t* cur = tokens + b * cap;
    int id, tid;
    sample_row(logits + b * (size_t)n_vocab, n_vocab, cur, i, i == 0, w.has_ts != 0, w.seek_delta, R, &id, &tid);
    if (threadIdx.x != 0) return;
    cur[i] = id;
    tids[b * cap + i] = tid;
    w.n_tokens = i + 1;
    const int window = 2 * R.n_audio_ctx;
    bool done = false;
    if (id > R.beg) {
        const int sd_new = 2 * (id - R.beg);
        if (w.has_ts && w.seek_delta > sd_new && w.result_len < i) {
            w.failed = 1;
            done = true;
        } else {
            w.seek_delta = sd_new;
            w.result_len = i + 1;
            w.has_ts = 1;
        }
    }
    if (!done && (id == R.eot || (w.has_ts && w.seek + w.seek_delta + 100 >= w.seek_end))) {
        if (w.result_len == 0) {
            if (w.seek + w.seek_delta + 100 >= w.seek_end)
                w.result_len = i + 1;
            else
                w.failed = 1;
        }
        done = true;
    }
    if (!done && i == n_max - 1 && (w.result_len == 0 || w.seek_delta < window / 2)) {
        w.failed = 1;
        done = true;
    }
    if (!done && i + 1 >= n_max) done = true;  // the loop runs out
    w.done = done ? 1 : 0;
    win[b] = w;
    next_token[b] = id;
}

}  // namespace ws
}  // namespace zwg

namespace {

int make_rules(const zwg_whisper_rules* r, zwg::ws::Rules* out) {
    if (!r) return fail("whisper rules: null");
    if (r->n_audio_ctx <= 0) return fail("whisper rules: n_audio_ctx must be positive");
    if (r->beg <= r->eot || r->eot <= 0) return fail("whisper rules: need 0 < eot < beg");
    if (r->n_hotwords < 0 || (r->n_hotwords > 0 && (!r->hotwords || !r->hotword_offsets)))
        return fail("whisper rules: hotwords need their token and offset arrays");
    zwg::ws::Rules R;
    R.eot = r->eot; R.sot = r->sot; R.translate = r->translate; R.transcribe = r->transcribe; R.solm = r->solm;
    R.prev = r->prev; R.nosp = r->nosp; R.not_ = r->not_; R.beg = r->beg; R.space = r->space;
    R.n_audio_ctx = r->n_audio_ctx;
    R.tid0_initial = -1;
    if (r->max_initial_ts > 0.f) {
        // src/transcribe.zig:521-523 in f32; @round rounds half away from zero, as roundf
        const float precision = 30.0f / (float)r->n_audio_ctx;
        R.tid0_initial = (int)roundf(r->max_initial_ts / precision);
    }
    R.hotword_bias = r->hotword_bias;
    R.hot_tokens = r->hotwords;
    R.hot_offsets = r->hotword_offsets;
    R.n_hot = r->n_hotwords;
    *out = R;
    return ZWG_OK;
}

}  // namespace

extern "C" {

int zwg_whisper_rules_default(zwg_whisper_rules* r) {
    if (!r) return fail("whisper rules: null");
    // src/model.zig:37-47 (English-only models), src/transcribe.zig:42-43, 94, 116
    r->eot = 50256; r->sot = 50257; r->translate = 50357; r->transcribe = 50358; r->solm = 50359;
    r->prev = 50360; r->nosp = 50361; r->not_ = 50362; r->beg = 50363; r->space = 220;
    r->n_audio_ctx = 1500;
    r->max_initial_ts = 1.0f;
    r->hotword_bias = 5.0f;
    r->hotwords = nullptr;
    r->hotword_offsets = nullptr;
    r->n_hotwords = 0;
    return ZWG_OK;
}

int zwg_whisper_sample(float* logits, size_t n_batch, size_t n_vocab, const int32_t* tokens, size_t tokens_stride,
                       const int32_t* n_tokens, const int32_t* has_ts, const int32_t* seek_delta,
                       const zwg_whisper_rules* rules, int32_t* out_id, int32_t* out_tid, void* stream) {
    zwg::ws::Rules R;
    int rc = make_rules(rules, &R);
    if (rc) return rc;
    if (n_batch == 0) return ZWG_OK;
    if (!logits || !out_id || !out_tid) return fail("whisper_sample: null logits or outputs");
    if (n_vocab <= (size_t)R.beg || n_vocab >= (1u << 30)) return fail("whisper_sample: n_vocab must exceed beg");
    if (n_tokens && !tokens) return fail("whisper_sample: n_tokens given without tokens");
    if (n_batch >= (1u << 31)) return fail("whisper_sample: batch too large");
    zwg::ws::whisper_sample_kernel<<<(unsigned)n_batch, zwg::ws::THREADS, 0, (cudaStream_t)stream>>>(
        logits, (int)n_vocab, tokens, tokens_stride, n_tokens, has_ts, seek_delta, R, out_id, out_tid);
    cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ZWG_OK : cuda_fail("whisper_sample launch", e);
}

int zwg_whisper_window_init(zwg_whisper_window* win, size_t n_batch, const zwg_whisper_rules* rules, void* stream) {
    zwg::ws::Rules R;
    int rc = make_rules(rules, &R);
    if (rc) return rc;
    if (n_batch == 0) return ZWG_OK;
    if (!win) return fail("whisper_window_init: null windows");
    const unsigned blocks = (unsigned)((n_batch + 255) / 256);
    zwg::ws::whisper_window_init_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(win, (int)n_batch, R.n_audio_ctx);
    cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ZWG_OK : cuda_fail("whisper_window_init launch", e);
}

int zwg_whisper_step(float* logits, size_t n_batch, size_t n_vocab, zwg_whisper_window* win, int32_t* tokens,
                     int32_t* tids, size_t cap, const zwg_whisper_rules* rules, size_t n_max, int32_t* next_token,
                     void* stream) {
    zwg::ws::Rules R;
    int rc = make_rules(rules, &R);
    if (rc) return rc;
    if (n_batch == 0) return ZWG_OK;
    if (!logits || !win || !tokens || !tids || !next_token) return fail("whisper_step: null buffer");
    if (n_vocab <= (size_t)R.beg || n_vocab >= (1u << 30)) return fail("whisper_step: n_vocab must exceed beg");
    if (n_max == 0 || n_max > cap || cap >= (1u << 30)) return fail("whisper_step: need 0 < n_max <= cap");
    zwg::ws::whisper_step_kernel<<<(unsigned)n_batch, zwg::ws::THREADS, 0, (cudaStream_t)stream>>>(
        logits, (int)n_vocab, win, tokens, tids, cap, R, (int)n_max, next_token);
    cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ZWG_OK : cuda_fail("whisper_step launch", e);
}

size_t zwg_whisper_decode_scratch_bytes(const zwg_dec_state* st, size_t n_vocab, size_t n_prompt) {
    if (!st || n_prompt == 0) return 0;
    const size_t al = 256;
    auto up = [&](size_t x) { return (x + al - 1) / al * al; };
    return up(st->n_batch * n_prompt * st->n_state * 4) + up(st->n_batch * n_vocab * 4) + up(st->n_batch * 4) +
           up(zwg_dec_scratch_bytes(st, n_prompt));
}

int zwg_whisper_decode_q8(zwg_dec_state* st, const zwg_dec_weights* w, const zwg_whisper_rules* rules,
                          const int32_t* prompt, size_t n_prompt, size_t n_max, zwg_whisper_window* win,
                          int32_t* tokens, int32_t* tids, size_t cap, size_t check_every, void* scratch,
                          size_t scratch_bytes, void* stream) {
    if (!st || !w) return fail("whisper_decode_q8: null state or weights");
    if (!prompt || n_prompt == 0) return fail("whisper_decode_q8: empty prompt");
    if (n_max == 0) n_max = st->n_text_ctx / 2 - 4;  // src/transcribe.zig:252
    if (n_max > cap) return fail("whisper_decode_q8: cap %zu < n_max %zu", cap, n_max);
    if (n_prompt + n_max - 1 > st->n_text_ctx)
        return fail("whisper_decode_q8: prompt %zu + %zu steps exceed the text context %zu", n_prompt, n_max,
                    st->n_text_ctx);
    if (!scratch || ((uintptr_t)scratch & 255)) return fail("whisper_decode_q8: scratch must be 256-byte aligned");
    const size_t need = zwg_whisper_decode_scratch_bytes(st, w->n_vocab, n_prompt);
    if (scratch_bytes < need) return fail("whisper_decode_q8: scratch %zu bytes, %zu needed", scratch_bytes, need);
    const size_t nb = st->n_batch;
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    uint8_t* p = static_cast<uint8_t*>(scratch);
    float* x = reinterpret_cast<float*>(p);
    p += up(nb * n_prompt * st->n_state * 4);
    float* logits = reinterpret_cast<float*>(p);
    p += up(nb * w->n_vocab * 4);
    int32_t* next = reinterpret_cast<int32_t*>(p);
    p += up(nb * 4);
    void* dscr = p;
    const size_t dscr_bytes = scratch_bytes - (size_t)(p - static_cast<uint8_t*>(scratch));
    const cudaStream_t s = (cudaStream_t)stream;
    int rc = zwg_whisper_window_init(win, nb, rules, stream);
    if (rc) return rc;
    // the prompt (src/transcribe.zig:293-294), then one token at a time (:316-362)
    if ((rc = zwg_dec_forward_q8(st, w, prompt, 0, n_prompt, x, logits, dscr, dscr_bytes, stream))) return rc;
    std::vector<zwg_whisper_window> host(nb);
    if (check_every == 0) check_every = n_max;
    for (size_t i = 0; i < n_max; i++) {
        if ((rc = zwg_whisper_step(logits, nb, w->n_vocab, win, tokens, tids, cap, rules, n_max, next, stream)))
            return rc;
        if ((i + 1) % check_every == 0 || i + 1 == n_max) {
            cudaError_t e = cudaMemcpyAsync(host.data(), win, nb * sizeof(zwg_whisper_window), cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) return cuda_fail("whisper_decode_q8: reading the windows' state", e);
            bool all = true;
            for (size_t b = 0; b < nb && all; b++) all = host[b].done != 0;
            if (all) break;
        }
        if (i + 1 < n_max && (rc = zwg_dec_forward_q8(st, w, next, n_prompt + i, 1, x, logits, dscr, dscr_bytes, stream)))
            return rc;
    }
    return ZWG_OK;
}

}  // extern "C"
