/*
 * zwgpu: B200 (sm_100a) attention engine for zwhisper, plain C ABI.
 *
 * Replaces the CPU attention routine of the reference, `ops.attentionEx`
 * (src/ops.zig:562-590), its MHA wrapper `ops.attention` (src/ops.zig:593-605) and the
 * scratch sizers (src/ops.zig:545-560), and adds device-resident entry points for the
 * four call sites: encoder self-attention (src/encoder.zig:167), decoder causal
 * self-attention (src/decoder.zig:184) and cross-attention (src/decoder.zig:191), and
 * Qwen2 grouped-query attention over a transposed key cache (src/llm.zig:178-202).
 *
 * Conventions (those of the reference's C ABI, include/zwhisper.h:33-75):
 *   - every function returns int: ZWG_OK (0), ZWG_ERROR (2), ZWG_TIMEOUT (4, a device-side
 *     wait gave up; the context stays usable); nothing traps or aborts;
 *   - the caller owns every buffer; entry points taking device pointers allocate nothing
 *     and take caller-sized workspace, like the reference's caller-sized scratch;
 *   - a context is per device and per calling thread: calls on one context are not
 *     re-entrant (the reference's handles are not thread-safe either, src/capi.zig:3-4).
 *     Run one host thread per device for multi-GPU sharding.
 * Strides and sizes are in elements. "bf16" buffers are uint16_t bit patterns.
 */
#ifndef ZWGPU_H
#define ZWGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define ZWG_API __attribute__((visibility("default")))
#else
#define ZWG_API
#endif

#define ZWG_OK 0
#define ZWG_ERROR 2
#define ZWG_TIMEOUT 4

/* Mirror of AttnShape (src/ops.zig:477-492). Query head h reads kv head
 * h / (n_head / n_head_kv). With causal set, query i sees keys j <= n_kv - n_q + i.
 * kt_stride == 0: keys are rows k[n_kv][kv_stride]; otherwise keys are kept transposed as
 * k[n_head_kv][d][kt_stride] (src/llm.zig:27-28), as in the reference's optional kt_stride. */
typedef struct zwg_attn_shape {
    size_t n_q;
    size_t n_kv;
    size_t n_head;
    size_t n_head_kv;
    size_t d;
    size_t q_stride;
    size_t kv_stride;
    size_t out_stride;
    int32_t causal;
    size_t kt_stride;
} zwg_attn_shape;

/* A batch of independent items (windows or sequences) sharing one shape; item b's
 * buffers start at base + b * *_batch_stride (elements). No reference counterpart: the
 * reference runs one window or sequence per call. */
typedef struct zwg_batch {
    size_t n_batch;
    size_t q_batch_stride;
    size_t k_batch_stride;
    size_t v_batch_stride;
    size_t out_batch_stride;
} zwg_batch;

/* Library version (the reference's zw_version, include/zwhisper.h:73, returns 3). */
ZWG_API int zwg_version(void);

/* Bind the calling thread to `device`, creating that device's context on first use
 * (stream, error word). Counterpart of the device set-up that zw_open adds
 * (src/capi.zig:59-79). */
ZWG_API int zwg_init(int device);

/* Release the calling thread's device context and its cached buffers. */
ZWG_API int zwg_shutdown(void);

/* Copy the last error message of the calling thread (NUL terminated, truncated to len).
 * Returns the full message length. */
ZWG_API size_t zwg_last_error(char* buf, size_t len);

/* Number of CUDA devices visible (0 when none). */
ZWG_API int zwg_device_count(void);

/* Math mode of the calling thread's context: ZWG_MATH_F32 (0, the default) or an OR of the
 * tensor-core flags below. No reference counterpart (the reference computes in f32 only).
 * ZWG_MATH_F32: f32 operands and accumulation on every shape, the reference's arithmetic.
 * ZWG_MATH_BF16 (host-pointer entry points): encoder-shaped calls (self-attention,
 *   n_q == n_kv, d == 64, MHA, rows of exactly n_head*64, keys as rows, not causal)
 *   convert Q/K/V to bf16 on the device and run the tcgen05 kernel with f32 softmax and
 *   accumulation.
 * ZWG_MATH_TF32 (host- and device-pointer entry points): calls over a transposed key cache
 *   (kt_stride > 0, d 64 or 128, 16-byte aligned buffers and strides that are multiples of
 *   4) run tcgen05 kernels with kind::tf32 operands read straight from the f32 caches
 *   (10-bit mantissa) and f32 softmax and accumulation: prefill-shaped calls (more than 8
 *   query rows per kv head) the prefill kernel, one-token calls with a GQA group of at most
 *   32 heads the split-K decode kernel. Other shapes stay f32. */
#define ZWG_MATH_F32 0
#define ZWG_MATH_BF16 1
#define ZWG_MATH_TF32 2
ZWG_API int zwg_set_math(int mode);

/* ---- drop-in, host pointers, synchronous (parity path) ------------------------------ */

/* ops.attentionEx (src/ops.zig:562): q[n_q][q_stride], k, v[n_kv][kv_stride],
 * out[n_q][out_stride], all host f32. Fills out before returning. The reference's
 * scratch argument is not needed: device staging is owned by the context. */
ZWG_API int zwg_attention(const zwg_attn_shape* sh, const float* q, const float* k, const float* v,
                  float* out);

/* ops.attention (src/ops.zig:593): MHA with q, k, v, out all [rows][n_state]. */
ZWG_API int zwg_attention_mha(const float* q, const float* k, const float* v, size_t n_q, size_t n_kv,
                      size_t n_state, size_t n_head, int32_t causal, float* out);

/* The same call over a batch of host items, pipelined (copies overlap compute). */
ZWG_API int zwg_attention_batch_host(const zwg_attn_shape* sh, const zwg_batch* b, const float* q,
                             const float* k, const float* v, float* out);

/* ---- device pointers, stream ordered (throughput path) ------------------------------- */

/* Workspace bytes zwg_attention_dev needs for this shape and batch (ops.attentionScratchEx,
 * src/ops.zig:545-556, sizes the reference's scratch the same way: per shape). */
ZWG_API size_t zwg_attention_workspace(const zwg_attn_shape* sh, const zwg_batch* b);

/* ops.attentionEx over a batch, device pointers. Decode-like shapes (n_q * n_head /
 * n_head_kv <= 8 rows per kv head) run the split-K kernel; others run the tiled f32
 * kernel, or the tf32 tensor-core kernel for the prefill shapes ZWG_MATH_TF32 covers.
 * `stream` is a cudaStream_t; NULL means the legacy default stream, as in the CUDA runtime. The device entry points below take `stream` the same way. */
ZWG_API int zwg_attention_dev(const zwg_attn_shape* sh, const zwg_batch* b, const float* q,
                      const float* k, const float* v, float* out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* No counterpart in the reference. The decode-shaped zwg_attention_dev (split-K kernel)
 * for callers that cannot allocate device memory: the split partials live in a 4 MiB
 * array inside the library instead of caller workspace, and the call allocates nothing.
 * Some hosts cannot call cudaMalloc: an embedding that reaches the engine only through
 * this C ABI from a runtime without CUDA allocator bindings, or a streaming decode thread
 * that must not stall, since cudaMalloc/cudaFree can synchronize the device. Limits and
 * rules: decode shapes only (d in {32, 64, 128}, n_q * n_head / n_head_kv <= 8); a call
 * whose partials exceed 4 MiB returns ZWG_ERROR with a message and launches nothing;
 * every device that loads the library holds the 4 MiB until exit; the first call on a
 * device looks up the array's device address (make it before any stream capture), and
 * the first call after a device reset looks it up again; all calls share the array, so
 * calls that overlap on the GPU race: keep one device's calls on one stream or ordered.
 * Shapes are checked as zwg_attention_dev checks them. Needs no zwg_init. */
ZWG_API int zwg_attention_dev_noalloc(const zwg_attn_shape* sh, const zwg_batch* b, const float* q,
                                      const float* k, const float* v, float* out, void* stream);

/* Encoder self-attention on tcgen05 tensor cores (src/encoder.zig:167): bf16 q, k, v
 * [n_batch][n_ctx][n_head*64], non-causal, d = 64, f32 softmax and accumulation,
 * f32 out [n_batch][n_ctx][n_head*64]. Rows of 16-byte aligned buffers are required
 * (TMA): q/k/v base addresses 16-byte aligned and n_head*64*2 bytes per row. */
ZWG_API int zwg_enc_attn_bf16(size_t n_batch, size_t n_ctx, size_t n_head, const uint16_t* q,
                      const uint16_t* k, const uint16_t* v, float* out, void* stream);

/* f32 -> bf16 (round to nearest even) of n elements, device pointers; the producer step
 * a projection epilogue would fuse. */
ZWG_API int zwg_f32_to_bf16(const float* x, uint16_t* y, size_t n, void* stream);

/* Qwen2 rotary embedding and cache append (src/llm.zig:182-190, 221-238): NeoX RoPE at
 * positions n_past.. on q[n][n_head*d] (in place) and k[n][n_head_kv*d], then
 * cache_kt[h][p][n_past+i] = k_rot[i][h*d+p] and cache_v[(n_past+i)][:] = v[i][:].
 * cos/sin tables are [n_ctx][d/2] f32 (computed in f64 on the host, src/llm.zig:128-137).
 * Batched: item b's q, k, v, cache_kt and cache_v start at b * the given strides. */
ZWG_API int zwg_rope_kt_append(size_t n_batch, size_t n, size_t n_past, size_t n_head, size_t n_head_kv,
                       size_t d, size_t n_ctx, float* q, const float* k, const float* v,
                       float* cache_kt, float* cache_v, const float* cos_tab,
                       const float* sin_tab, size_t q_bstride, size_t kv_bstride,
                       size_t cache_bstride, void* stream);

/* ---- Q8 weights: the projections around the attention calls ------------------------ */

/* gemm.Q8.quantize (src/gemm.zig:208-230) on the device: w [n][k] f32 (k a multiple of 32)
 * -> q [n][k] int8 and scales [n][k/32] f32, scale = absmax / 127 per block of 32 and q =
 * clamp(round(w * 127 / absmax), -127, 127): bit-identical to the reference. */
ZWG_API int zwg_q8_quantize(const float* w, size_t n, size_t k, int8_t* q, float* scales, void* stream);

/* ops.linear with Q8 weights (src/ops.zig:280-306 -> gemm.ntBlockQ, src/gemm.zig:268-351):
 * out[m][n] = x[m][k] . W[n][k]^T + bias[n], W = q * scale per block of 32; bias may be NULL.
 * Device pointers; x [m][k] and out [m][n] f32 row-major, k a multiple of 32, x and q
 * 16-byte aligned. f32 arithmetic; up to 15 rows of x stream the weight bytes once per 8
 * rows, 16 or more run as a tiled product (the weights read once per tile): on the tcgen05
 * tensor cores when k is a multiple of 64 (each 32-wide block dot formed exactly from int8
 * weights and three bf16 pieces of each activation, then scaled as the reference does),
 * else on a register-tiled CUDA-core kernel. */
ZWG_API int zwg_linear_q8(const float* x, size_t m, size_t k, const int8_t* q, const float* scales,
                          const float* bias, size_t n, float* out, void* stream);

/* Where the Q8 products of 16 or more rows with k a multiple of 64 (zwg_linear_q8, the
 * decoder / LLM projections, the SiLU pair and the q/k/v products) run: 1 (the default) on
 * the tcgen05 kernel except small products at up to 64 rows (k <= 1024 and at most 1.25 M
 * weights, faster on the CUDA-core kernel), 2 on the tcgen05 kernel for every such
 * product, 0 on the register-tiled CUDA-core kernel. Process-wide; returns the previous
 * setting; a negative argument only queries it. */
ZWG_API int zwg_q8_tensor_cores(int enable);

/* ---- library-owned device state (the device-resident API) ---------------------------
 * The reference keeps its attention buffers inside the decoder and the LLM
 * (src/decoder.zig:39-42, 127-130; src/llm.zig:27-28, 124-137). These states hold the
 * same buffers on the device for n_batch windows or sequences, so a GPU-resident caller
 * passes only the new rows and the queries. States are created on the calling thread's
 * device (zwg_init) and used from threads bound to that device; calls are stream ordered
 * (`stream` as above). q, k_new, v_new, out and the LLM's q/k/v are device pointers;
 * zwg_cross_kv_set also takes host pointers (pinned for an asynchronous copy). Buffers
 * are batched: item b of q/out/k_new/v_new starts at b times one item's size. */

/* Whisper decoder: per layer a self K/V cache [n_batch][n_text_ctx][n_state] and cross
 * K/V [n_batch][n_audio_ctx][n_state]. */
typedef struct zwg_dec_state zwg_dec_state;
ZWG_API int zwg_dec_state_create(size_t n_layer, size_t n_batch, size_t n_state, size_t n_head,
                                 size_t n_text_ctx, size_t n_audio_ctx, zwg_dec_state** out);
ZWG_API int zwg_dec_state_destroy(zwg_dec_state* st);
/* Device pointers of one layer's buffers (any output may be NULL). */
ZWG_API int zwg_dec_state_cache(const zwg_dec_state* st, size_t layer, float** self_k, float** self_v,
                                float** cross_k, float** cross_v);
/* setAudio (src/decoder.zig:150-156) for one window and layer: k, v [n_audio_ctx][n_state]. */
ZWG_API int zwg_cross_kv_set(zwg_dec_state* st, size_t layer, size_t window, const float* k,
                             const float* v, void* stream);
/* One decoder step's attention for every window (src/decoder.zig:179-191), q and out
 * [n_batch][n][n_state]. ZWG_DEC_SELF: k_new, v_new [n_batch][n][n_state] are written at
 * rows n_past.. of the layer's cache, then causal attention over n_past + n keys; with both
 * NULL those rows are taken as already written (by a kernel of the caller's on the same
 * stream, through zwg_dec_state_cache's pointers).
 * ZWG_DEC_CROSS: attention over the window's cross K/V (k_new, v_new, n_past unused). */
#define ZWG_DEC_SELF 0
#define ZWG_DEC_CROSS 1
ZWG_API int zwg_dec_step_attn(zwg_dec_state* st, size_t layer, int kind, const float* q, const float* k_new,
                              const float* v_new, size_t n_past, size_t n, float* out, void* stream);

/* Qwen2 LLM: per layer cache_kt [n_batch][n_head_kv][d][n_ctx] (zeroed) and cache_v
 * [n_batch][n_ctx][n_head_kv*d]; RoPE tables [n_ctx][d/2] computed in f64 and cast to f32
 * with base rope_base (src/llm.zig:128-137). */
typedef struct zwg_llm_state zwg_llm_state;
ZWG_API int zwg_llm_state_create(size_t n_layer, size_t n_batch, size_t n_head, size_t n_head_kv, size_t d,
                                 size_t n_ctx, double rope_base, zwg_llm_state** out);
ZWG_API int zwg_llm_state_destroy(zwg_llm_state* st);
ZWG_API int zwg_llm_state_cache(const zwg_llm_state* st, size_t layer, float** cache_kt, float** cache_v);
/* RoPE and cache append (src/llm.zig:180-190): q [n_batch][n][n_head*d] rotated in place;
 * k, v [n_batch][n][n_head_kv*d] rotated (k) and written at positions n_past.. */
ZWG_API int zwg_llm_append_rope(zwg_llm_state* st, size_t layer, float* q, const float* k, const float* v,
                                size_t n_past, size_t n, void* stream);
/* Causal GQA attention of q [n_batch][n][n_head*d] over the layer's cache, n_kv = n_past + n
 * (src/llm.zig:191-202); out as q. The context's math mode applies (ZWG_MATH_TF32 runs
 * prefill chunks on tensor cores). _decode is the n = 1 call. */
ZWG_API int zwg_llm_attn_prefill(zwg_llm_state* st, size_t layer, const float* q, size_t n_past, size_t n,
                                 float* out, void* stream);
ZWG_API int zwg_llm_attn_decode(zwg_llm_state* st, size_t layer, const float* q, size_t n_past, float* out,
                                void* stream);

/* ---- the Qwen2 decode step around the attention (src/llm.zig:168-216, 268-321) --------
 * The rest of Model.forward, so a greedy decode keeps hidden states, caches and tokens on
 * the device. All buffers are device pointers; calls are stream ordered. The projection,
 * norm and sampling kernels start early when they follow one another on a stream: each
 * streams its own weights while the kernel before it finishes, and reads that kernel's
 * results only once it has completed. Q8 matrices are int8 [n][k] plus f32 scales
 * [n][k/32] (gemm.Q8, src/gemm.zig:188-200). */
typedef struct zwg_q8_mat {
    const int8_t* q;
    const float* scales;
} zwg_q8_mat;

/* One layer's weights (llm.Layer, src/llm.zig:15-30, without the caches): attn_norm and
 * ffn_norm [n_embd]; wq [n_head*d][n_embd]; wk, wv [n_head_kv*d][n_embd]; wo
 * [n_embd][n_head*d]; w_gate, w_up [n_ff][n_embd]; w_down [n_embd][n_ff]. bq, bk, bv are
 * f32 or NULL. */
typedef struct zwg_llm_layer_weights {
    const float* attn_norm;
    zwg_q8_mat wq, wk, wv, wo;
    const float* bq;
    const float* bk;
    const float* bv;
    const float* ffn_norm;
    zwg_q8_mat w_gate, w_up, w_down;
} zwg_llm_layer_weights;

/* The model's weights (llm.Model, src/llm.zig:32-60): embd and output [n_vocab][n_embd] (the
 * same matrix when tied), output_norm [n_embd], `layers` a HOST array of the state's n_layer
 * entries. n_embd must equal n_head * d, as the reference's buffers assume; n_embd and n_ff
 * are multiples of 32. */
typedef struct zwg_llm_weights {
    size_t n_vocab, n_embd, n_ff;
    float eps;
    zwg_q8_mat embd, output;
    const float* output_norm;
    const zwg_llm_layer_weights* layers;
} zwg_llm_weights;

/* ops.rmsNorm (src/ops.zig:408-425): out[i] = x[i] * (1 / sqrt(mean(x[i]^2) + eps)) * w for
 * m rows of n (n a multiple of 4, 16-byte aligned buffers); out may be x. */
ZWG_API int zwg_rms_norm(const float* x, size_t m, size_t n, const float* w, float eps, float* out, void* stream);

/* ops.linear then ops.add (src/llm.zig:203-204, 209-210): out[m][n] += x[m][k] . W^T, with
 * W Q8 as zwg_linear_q8 (the residual stream updated in place). */
ZWG_API int zwg_linear_q8_add(const float* x, size_t m, size_t k, const int8_t* q, const float* scales, size_t n,
                              float* out, void* stream);

/* The gate and up projections and ops.siluMul (src/llm.zig:206-208, src/ops.zig:435-440) in
 * one launch: out[m][n] = silu(x . Wg^T) * (x . Wu^T), silu(g) = g / (1 + exp(-g)). */
ZWG_API int zwg_linear_q8_silu_mul(const float* x, size_t m, size_t k, const int8_t* gate_q,
                                   const float* gate_scales, const int8_t* up_q, const float* up_scales, size_t n,
                                   float* out, void* stream);

/* Q8.row (src/gemm.zig:256-263) for each token: out[i][:] = q[tokens[i]][:] * scales, the
 * embedding lookup of src/llm.zig:175, bit-identical. A token outside [0, n_vocab) gives a
 * zero row and sets the device error word (reported by zwg_sync). */
ZWG_API int zwg_embed_q8(const int32_t* tokens, size_t m, const int8_t* q, const float* scales, size_t n_vocab,
                         size_t k, float* out, void* stream);

/* Model.penalize then Model.argmax (src/llm.zig:268-273, 313-321) for m rows of logits
 * [m][n_vocab], in place: when penalty > 1, the logits of row i's last `window` entries
 * of recent[i * recent_stride + 0 .. n_recent) are divided by penalty (positive) or
 * multiplied by it (otherwise), repeats again each time; then out[i * out_stride] = the
 * first index of the largest logit. */
ZWG_API int zwg_llm_greedy(float* logits, size_t m, size_t n_vocab, const int32_t* recent, size_t recent_stride,
                           size_t n_recent, size_t window, float penalty, int32_t* out, size_t out_stride,
                           void* stream);

/* The q, k and v projections with their biases, RoPE at positions n_past.. and the cache
 * append (src/llm.zig:179-190) in one launch: x [n_batch][n][n_head*d] (the normed hidden
 * states) -> q_out [n_batch][n][n_head*d] rotated, k rotated into the layer's cache_kt and v
 * into its cache_v. Uses w->wq, wk, wv, bq, bk, bv. */
ZWG_API int zwg_llm_qkv_q8(zwg_llm_state* st, size_t layer, const float* x, const zwg_llm_layer_weights* w,
                           size_t n_past, size_t n, float* q_out, void* stream);

/* Scratch bytes zwg_llm_layer_q8 and zwg_llm_forward_q8 need for chunks of n tokens. */
ZWG_API size_t zwg_llm_scratch_bytes(const zwg_llm_state* st, size_t n, size_t n_ff);

/* One layer of Model.forward (src/llm.zig:177-210) for every sequence: x [n_batch][n][n_embd],
 * the residual stream, updated in place; tokens at positions n_past..n_past+n-1. Runs
 * rmsNorm, zwg_llm_qkv_q8, the attention (as zwg_llm_attn_prefill), wo + residual,
 * rmsNorm, gate/up + siluMul, w_down + residual. */
ZWG_API int zwg_llm_layer_q8(zwg_llm_state* st, size_t layer, const zwg_llm_weights* w, float* x, size_t n_past,
                             size_t n, void* scratch, size_t scratch_bytes, void* stream);

/* Model.forward (src/llm.zig:169-216) for every sequence: tokens [n_batch][n] (device int32)
 * at positions n_past.., hidden states left in x [n_batch][n][n_embd], and the logits of
 * each sequence's last token in logits [n_batch][n_vocab]. */
ZWG_API int zwg_llm_forward_q8(zwg_llm_state* st, const zwg_llm_weights* w, const int32_t* tokens, size_t n_past,
                               size_t n, float* x, float* logits, void* scratch, size_t scratch_bytes,
                               void* stream);

/* ---- the Whisper decoder step on the device (src/decoder.zig:150-206) -----------------
 * Decoder.forward and setAudio around the state's attention calls, for n_batch windows:
 * LayerNorm, Q8 projections with their biases, GELU, the residual adds, the token and
 * position embeddings and the tied logits. Q8 matrices as zwg_q8_mat; vectors f32 [n_state]
 * (mlp0_b [4 n_state]); all device pointers. */
typedef struct zwg_dec_layer_weights {
    const float* attn_ln_w;
    const float* attn_ln_b;
    zwg_q8_mat q;               /* [n_state][n_state] */
    const float* q_b;
    zwg_q8_mat k;               /* no bias, as the model */
    zwg_q8_mat v;
    const float* v_b;
    zwg_q8_mat o;
    const float* o_b;
    const float* cross_ln_w;
    const float* cross_ln_b;
    zwg_q8_mat cq;
    const float* cq_b;
    zwg_q8_mat ck;              /* no bias */
    zwg_q8_mat cv;
    const float* cv_b;
    zwg_q8_mat co;
    const float* co_b;
    const float* mlp_ln_w;
    const float* mlp_ln_b;
    zwg_q8_mat mlp0;            /* [4 n_state][n_state] */
    const float* mlp0_b;
    zwg_q8_mat mlp1;            /* [n_state][4 n_state] */
    const float* mlp1_b;
} zwg_dec_layer_weights;

/* The decoder's weights (decoder.Decoder, src/decoder.zig:45-60): te [n_vocab][n_state] (the
 * token embedding and the tied logits matrix), pe [n_text_ctx][n_state], the final LayerNorm,
 * `layers` a HOST array of the state's n_layer entries. n_state a multiple of 32. */
typedef struct zwg_dec_weights {
    size_t n_vocab;
    zwg_q8_mat te;
    const float* pe;
    const float* ln_w;
    const float* ln_b;
    const zwg_dec_layer_weights* layers;
} zwg_dec_weights;

/* ops.layerNorm (src/ops.zig:355-398): out[i] = (x[i] - mean) / sqrt(var + eps) * w + b for m
 * rows of n (population variance; n a multiple of 4, 16-byte aligned buffers). */
ZWG_API int zwg_layer_norm(const float* x, size_t m, size_t n, const float* w, const float* b, float eps, float* out,
                           void* stream);

/* ops.linear then ops.gelu (src/decoder.zig:197-198): out[m][n] = gelu(x . W^T + bias), ggml's
 * tanh GELU (src/ops.zig:312-327). */
ZWG_API int zwg_linear_q8_gelu(const float* x, size_t m, size_t k, const int8_t* q, const float* scales,
                               const float* bias, size_t n, float* out, void* stream);

/* setAudio (src/decoder.zig:151-159) for one window: enc [n_audio_ctx][n_state] (device) ->
 * every layer's cross K = enc . ck^T and cross V = enc . cv^T + cv_b in the state. */
ZWG_API int zwg_dec_set_audio_q8(zwg_dec_state* st, const zwg_dec_weights* w, size_t window, const float* enc,
                                 void* stream);

/* Scratch bytes zwg_dec_forward_q8 needs for chunks of n tokens. */
ZWG_API size_t zwg_dec_scratch_bytes(const zwg_dec_state* st, size_t n);

/* Decoder.forward (src/decoder.zig:166-206) for every window: tokens [n_batch][n] (device
 * int32) at positions n_past..; hidden states left in x [n_batch][n][n_state]; the logits of
 * each window's last token in logits [n_batch][n_vocab]. The self K/V rows are appended to
 * the state's cache; cross-attention reads the state's cross K/V (zwg_cross_kv_set or
 * zwg_dec_set_audio_q8). */
ZWG_API int zwg_dec_forward_q8(zwg_dec_state* st, const zwg_dec_weights* w, const int32_t* tokens, size_t n_past,
                               size_t n, float* x, float* logits, void* scratch, size_t scratch_bytes, void* stream);

/* ---- Whisper's greedy decoding rules on the device (src/transcribe.zig:176-193, 248-580) ---
 * The transcription driver's per-token sampling (Engine.sample) and the bookkeeping of its
 * window loop, so a window's tokens stay on the device between decoder steps. */

/* Special token ids and options of Engine.sample: the ids of src/model.zig:37-47 (`space`
 * is the id of the token " ", src/transcribe.zig:116), n_audio_ctx (30 s = 2 * n_audio_ctx
 * mel frames), max_initial_ts in seconds (<= 0 turns the rule off, Options.max_initial_ts),
 * hotword_bias (Engine.hotword_bias) and the hotword forms as DEVICE arrays: the forms'
 * token ids concatenated in `hotwords`, form f at [hotword_offsets[f], hotword_offsets[f+1])
 * (n_hotwords + 1 offsets; each hotword's two forms, with and without a leading space, in
 * the reference's order). */
typedef struct zwg_whisper_rules {
    int32_t eot, sot, translate, transcribe, solm, prev, nosp, not_, beg, space;
    int32_t n_audio_ctx;
    float max_initial_ts;
    float hotword_bias;
    const int32_t* hotwords;
    const int32_t* hotword_offsets;
    int32_t n_hotwords;
} zwg_whisper_rules;

/* The reference's defaults for English-only models: the ids above, n_audio_ctx 1500,
 * max_initial_ts 1 s, hotword bias 5, no hotwords. */
ZWG_API int zwg_whisper_rules_default(zwg_whisper_rules* r);

/* Engine.sample (src/transcribe.zig:491-580) for n_batch rows of logits [n_batch][n_vocab]
 * (device f32, modified in place as the reference modifies Engine.logits): row b's window
 * has sampled tokens[b * tokens_stride + 0 .. n_tokens[b]) so far (device int32; n_tokens
 * NULL: none, the first token), has_ts[b] and seek_delta[b] of the window loop (NULL: 0 and
 * 2 * n_audio_ctx). out_id[b] = the chosen token, out_tid[b] = the most likely timestamp
 * (device int32). The token ids equal the reference's; the log-sum-exp sums agree to f32
 * rounding. */
ZWG_API int zwg_whisper_sample(float* logits, size_t n_batch, size_t n_vocab, const int32_t* tokens,
                               size_t tokens_stride, const int32_t* n_tokens, const int32_t* has_ts,
                               const int32_t* seek_delta, const zwg_whisper_rules* rules, int32_t* out_id,
                               int32_t* out_tid, void* stream);

/* One window's state in the token loop of Engine.transcribe (src/transcribe.zig:292-365), in
 * device memory. The caller sets seek (the window's first mel frame) and seek_end (mel frames
 * of audio present, Mel.n_len_org); zwg_whisper_window_init sets the rest. After the loop:
 * the result is tokens[0 .. result_len), the next window starts seek_delta frames later,
 * failed with result_len 0 means nothing usable (the reference then moves on by a whole
 * window). */
typedef struct zwg_whisper_window {
    int32_t seek;
    int32_t seek_end;
    int32_t n_tokens;     /* tokens sampled so far */
    int32_t seek_delta;
    int32_t has_ts;
    int32_t result_len;
    int32_t failed;
    int32_t done;         /* the loop has ended for this window */
} zwg_whisper_window;

ZWG_API int zwg_whisper_window_init(zwg_whisper_window* win, size_t n_batch, const zwg_whisper_rules* rules,
                                    void* stream);

/* One step of the loop for every window that has not ended: Engine.sample on its logits row,
 * then the loop body's bookkeeping (src/transcribe.zig:319-364): the token and the best
 * timestamp appended at tokens/tids[b * cap + n_tokens] (device int32), seek_delta, has_ts,
 * result_len, failed and done updated. next_token[b] (device int32) is the decoder's next
 * input; a window that has ended keeps its last token there. n_max: the loop's token limit
 * (n_text_ctx / 2 - 4 in the reference), at most cap. */
ZWG_API int zwg_whisper_step(float* logits, size_t n_batch, size_t n_vocab, zwg_whisper_window* win, int32_t* tokens,
                             int32_t* tids, size_t cap, const zwg_whisper_rules* rules, size_t n_max,
                             int32_t* next_token, void* stream);

/* Scratch bytes zwg_whisper_decode_q8 needs for a prompt of n_prompt tokens. */
ZWG_API size_t zwg_whisper_decode_scratch_bytes(const zwg_dec_state* st, size_t n_vocab, size_t n_prompt);

/* The whole token loop of one window for each of the state's n_batch windows, on the device:
 * Decoder.forward of the prompt [n_batch][n_prompt] (device int32; the windows share its
 * length), then up to n_max (0: n_text_ctx / 2 - 4) steps of zwg_whisper_step and
 * zwg_dec_forward_q8. Tokens never leave the device; the host reads the windows' states
 * (n_batch * 32 bytes) every check_every steps (0: only at the end) and stops once every
 * window is done. The cross K/V must be set (zwg_dec_set_audio_q8) and win[b].seek, seek_end
 * filled; on return win, tokens and tids [n_batch][cap] hold each window's loop as the
 * reference leaves it. Synchronizes `stream`. */
ZWG_API int zwg_whisper_decode_q8(zwg_dec_state* st, const zwg_dec_weights* w, const zwg_whisper_rules* rules,
                                  const int32_t* prompt, size_t n_prompt, size_t n_max, zwg_whisper_window* win,
                                  int32_t* tokens, int32_t* tids, size_t cap, size_t check_every, void* scratch,
                                  size_t scratch_bytes, void* stream);

/* ---- Whisper encoder on the device (src/encoder.zig:118-179) ----------------------------
 * f16 weights as in the model file (exact in f16); every product on tcgen05 tensor cores with
 * f16 operands (activations rounded to f16) and f32 accumulation; attention on the bf16
 * kernel of zwg_enc_attn_bf16; LayerNorm, biases, GELU, residual adds and the positional
 * embedding in f32. Weight matrices are f16 [n_out][n_in] row-major (the file's layout);
 * vectors f32; all device pointers, 16-byte aligned. */
typedef struct zwg_enc_layer_weights {
    const float* attn_ln_w;
    const float* attn_ln_b;
    const uint16_t* w_qkv;      /* [3 n_state][n_state]: query, key and value rows stacked */
    const float* b_qkv;         /* [3 n_state]: query bias, zeros (the key has none), value bias */
    const uint16_t* w_o;        /* [n_state][n_state] */
    const float* b_o;
    const float* mlp_ln_w;
    const float* mlp_ln_b;
    const uint16_t* w_mlp0;     /* [4 n_state][n_state] */
    const float* b_mlp0;
    const uint16_t* w_mlp2;     /* [n_state][4 n_state] */
    const float* b_mlp2;
} zwg_enc_layer_weights;

/* The encoder's weights (Encoder, src/encoder.zig:12-40). The convolution weights are
 * stored tap-major: row n of conv1_w is [3][n_mels] (taps k = 0, 1, 2 of every mel channel,
 * the file's [n_mels][3] transposed), row n of conv2_w is [3][n_state]. pos [n_ctx][n_state];
 * `layers` a HOST array of n_layer entries. n_state a multiple of 128 (at most 1024) with
 * n_head = n_state / 64; n_mels a multiple of 8. */
typedef struct zwg_enc_weights {
    size_t n_mels, n_ctx, n_state, n_head, n_layer;
    const uint16_t* conv1_w;    /* [n_state][3 n_mels] */
    const float* conv1_b;
    const uint16_t* conv2_w;    /* [n_state][3 n_state] */
    const float* conv2_b;
    const float* pos;
    const zwg_enc_layer_weights* layers;
    const float* ln_post_w;
    const float* ln_post_b;
} zwg_enc_weights;

/* mel.logMel (src/mel.zig:103-157) on the device: samples [n_samples] f32 (16 kHz), filters
 * [n_mel][201] f32 (the model file's mel filters), out [n_mel][zwg_mel_frames(n_samples)]
 * f32: 200 samples reflected at the front, 30 s of zeros appended, 400-sample Hann frames
 * every 160 samples, DFT power, mel sums in f64, log10 with a 1e-10 floor, clamp to max - 8,
 * (x + 4) / 4. The DFT sums run in f32 in another order than the reference's radix-2 FFT, so
 * values agree to f32 rounding. scratch: zwg_mel_scratch_bytes() bytes of device memory. */
ZWG_API size_t zwg_mel_frames(size_t n_samples);
ZWG_API size_t zwg_mel_scratch_bytes(void);
ZWG_API int zwg_log_mel(const float* samples, size_t n_samples, const float* filters, size_t n_mel, float* out,
                        void* scratch, size_t scratch_bytes, void* stream);

/* Scratch bytes zwg_enc_forward_f16 needs for n_windows windows. */
ZWG_API size_t zwg_enc_scratch_bytes(const zwg_enc_weights* w, size_t n_windows);

/* Encoder.forward (src/encoder.zig:118-179) for n_windows windows of 2 n_ctx mel frames:
 * mel [n_mels][n_len] f32 (device), window i starting at frame offsets[i] (device int32
 * array; NULL: i * 2 n_ctx); out [n_windows][n_ctx][n_state] f32 (device), the encoder
 * output after ln_post. Launches only; the stream orders it. */
ZWG_API int zwg_enc_forward_f16(const zwg_enc_weights* w, const float* mel, size_t n_len, const int32_t* offsets,
                                size_t n_windows, float* out, void* scratch, size_t scratch_bytes, void* stream);

/* One f16 GEMM on the tensor cores, the encoder's building block (ops.linear, src/ops.zig:
 * 243-306, with f16 weights): for b < n_batch, m < M, n < N,
 *   v = sum_k a[b*a_bs + m*lda + k] * w[n*ldw + k] + bias[n]; gelu: v = gelu_tanh(v);
 *   addend: v += addend[m*ld_add + n]; accumulate: v += out[...];
 *   out[b*out_bs + m*ld_out + n] = v as out_type (ZWG_GEMM_F32 / F16 / BF16).
 * a, w f16; bias, addend f32 or NULL. N a multiple of 32, K, lda, ldw, a_bs multiples of 8;
 * rows of `a` may overlap (lda < K), which the encoder's convolutions use. */
#define ZWG_GEMM_F32 0
#define ZWG_GEMM_F16 1
#define ZWG_GEMM_BF16 2
ZWG_API int zwg_gemm_f16(const uint16_t* a, size_t lda, size_t a_bs, const uint16_t* w, size_t ldw, size_t M, size_t N,
                         size_t K, size_t n_batch, const float* bias, int gelu, const float* addend, size_t ld_add,
                         int accumulate, void* out, int out_type, size_t ld_out, size_t out_bs, void* stream);

/* Self-test of the timeout path every kernel relies on: launches one bounded device-side
 * wait on a barrier nothing ever completes (a few seconds), then synchronizes. Returns
 * ZWG_TIMEOUT when the wait ran out, was reported through the error word and left the
 * context usable (the expected result); ZWG_ERROR otherwise. No reference counterpart. */
ZWG_API int zwg_selftest_timeout(void);

/* Synchronize the device and report the context's device-side error word, if set. */
ZWG_API int zwg_sync(void);

#ifdef __cplusplus
}
#endif
#endif
