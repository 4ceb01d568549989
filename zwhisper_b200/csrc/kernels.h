// Internal kernel parameter blocks and launchers shared by the C-ABI layer (api.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace zwg {

// Batched attentionEx arguments (the AttnShape fields of src/ops.zig:477-492 plus
// per-item strides). Strides are in elements.
struct FlashParams {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    size_t n_q, n_kv, n_head, n_head_kv, d;
    size_t q_stride, kv_stride, out_stride;
    size_t kt_stride;  // 0: keys are rows
    int causal;
    size_t q_bs, k_bs, v_bs, out_bs;
};

struct DecodeParams {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    float* ws;  // split partials [n_batch][n_head_kv][n_splits][rows][d + 2]
    size_t n_q, n_kv, n_head, n_head_kv, d;
    size_t q_stride, kv_stride, out_stride;
    size_t kt_stride;
    int causal;
    int n_splits;
    int chunk;  // keys per split
    size_t q_bs, k_bs, v_bs, out_bs;
    // Segment tickets of the split decode kernels, n_batch * n_head_kv ints that are zero
    // at launch; the last CTA of each segment puts its ticket back to zero, so a buffer the
    // caller keeps for this alone needs no clearing between calls. nullptr: the tickets
    // follow the partials in ws and are cleared on the stream before the kernel.
    int* tickets;
};

int flash_f32_launch(const FlashParams& p, size_t n_batch, cudaStream_t st);

// Record the calling thread's last error message (read by zwg_last_error); return ZWG_ERROR.
int set_last_error(const char* msg);
int set_last_error_cuda(const char* what, cudaError_t e);

bool decode_supported(size_t d, size_t rows, size_t kt_stride);
void decode_plan(size_t n_batch, size_t n_head_kv, size_t n_kv, bool kt, int sm_count,
                 int* n_splits, int* chunk);
size_t decode_workspace_floats(size_t n_batch, size_t n_head_kv, size_t rows, int n_splits, size_t d);
int decode_f32_launch(const DecodeParams& p, size_t n_batch, cudaStream_t st);
int decode_combine_launch(const DecodeParams& p, size_t n_batch, cudaStream_t st);

// TMA-fed, stream-K scheduled decode kernel (attn_decode_tma.cu).
bool decode_tma_supported(const DecodeParams& p);
void decode_tma_plan(size_t n_batch, size_t n_head_kv, size_t n_kv, int sm_count, int* grid, int* p_max);
size_t decode_tma_workspace_bytes(size_t n_batch, size_t n_head_kv, size_t rows, size_t d, int p_max);
int decode_tma_launch(const DecodeParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st);

// Qwen2 decode on tcgen05 tensor cores, kind::tf32 over the transposed f32 key cache, split
// over the keys (attn_decode_tc.cu): one query token, d 64 or 128, group <= 32.
bool decode_tc_supported(const DecodeParams& p, size_t n_batch);
size_t decode_tc_workspace_bytes(size_t n_batch, size_t n_head_kv, size_t group, size_t d);
int decode_tc_launch(const DecodeParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st);

// Encoder tensor-core attention (attn_tc.cu).
struct EncTcParams {
    const uint16_t* q;
    const uint16_t* k;
    const uint16_t* v;
    float* out;
    int n_batch, n_ctx, n_head;
    int* err;  // device error word
    // Row stride of q, k and v in elements (0: n_head * 64, dense rows); a fused q|k|v
    // projection output passes 3 * n_state.
    size_t ld_qkv;
    // Non-zero: out is f16 [n_batch][n_ctx][n_head * 64] (the next projection's operand)
    // instead of f32.
    int out_f16;
};
int enc_tc_launch(const EncTcParams& p, cudaStream_t st);

// ---- f16 GEMM on tcgen05 (gemm_tc.cu): the encoder's projections and convolutions --------
enum { GEMM_OUT_F32 = 0, GEMM_OUT_F16 = 1, GEMM_OUT_BF16 = 2 };
struct GemmEpilogue {
    const float* bias;    // [N], or nullptr
    const float* addend;  // [M][ld_add] f32 added after the activation (the same for every
                          // batch: the positional embedding), or nullptr
    size_t ld_add;
    void* out;            // [batch][M][N] at ld_out per row, out_bs per batch (elements)
    size_t ld_out, out_bs;
};
struct GemmParams {
    const uint16_t* a;    // f16 [batch][M][K]: row m of batch b at a + b * a_bs + m * lda
    size_t lda, a_bs;     // a_bs 0: lda * M
    const uint16_t* w;    // f16 [N][K], row stride ldw
    size_t ldw;
    int M, N, K, n_batch;
    int out_type;         // GEMM_OUT_*
    bool gelu;            // tanh GELU after the bias
    bool accumulate;      // out (f32) += result
    GemmEpilogue e;
};
bool gemm_f16_supported(const GemmParams& p);
int gemm_f16_launch(const GemmParams& p, int sm_count, int* err, cudaStream_t st);

// ---- encoder helpers (enc_aux.cu) -----------------------------------------------------------
// LayerNorm of n_rows rows of n f32 (n a multiple of 128, at most 1024), one warp per row;
// out f16 (out_f16) or f32, which may be x itself.
int layer_norm_rows_launch(const float* x, size_t n_rows, int n, const float* w, const float* b, float eps, void* out,
                           bool out_f16, cudaStream_t st);
// Mel frames of each window as f16 rows: rows[b][1 + t][c] = mel[c][off_b + t] for t < n_frames
// (zero past n_len), rows[b][0] and rows[b][n_frames + 1] zero; off_b = offsets[b], or
// b * n_frames when offsets is null.
// ---- log-mel spectrogram (mel.cu) ----------------------------------------------------------
// Frames of the spectrogram of n samples (the reference's n_len, 30 s of zero pad included).
size_t mel_frames(size_t n_samples);
size_t mel_scratch_bytes();
// out [n_mel][mel_frames(n)] from samples [n] and filters [n_mel][201] (device pointers).
int log_mel_launch(const float* samples, size_t n, const float* filters, int n_mel, float* out, void* scratch,
                   int sm_count, cudaStream_t st);
int mel_rows_launch(const float* mel, int n_mels, size_t n_len, const int* offsets, int n_batch, int n_frames,
                    uint16_t* rows, cudaStream_t st);

// Prefill over a transposed key cache on tcgen05 tensor cores, kind::tf32
// (attn_prefill_tc.cu): d 64 or 128, group <= 128, TMA-aligned buffers and strides.
bool prefill_tc_supported(const FlashParams& p, size_t n_batch);
int prefill_tc_launch(const FlashParams& p, size_t n_batch, int sm_count, int* err, cudaStream_t st);

// Q8 weights (q8.cu): Q8.quantize and ops.linear over int8 blocks of 32.
int q8_quantize_launch(const float* w, size_t n, size_t k, int8_t* q, float* scales, cudaStream_t st);
// out = x . W^T (+ bias), then by mode: LIN_STORE writes it, LIN_ADD adds it into out (the
// residual), LIN_GELU writes gelu of it.
enum { LIN_STORE = 0, LIN_ADD = 1, LIN_GELU = 2 };
int q8_linear_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias,
                     size_t n, int mode, float* out, cudaStream_t st);

// Paired-row Q8 products with a fused epilogue (q8.cu): PAIR_ROPE = the q/k/v projections
// with bias, RoPE and the K^T / V cache append; PAIR_SILU = silu(x . Wg^T) * (x . Wu^T).
enum { PAIR_ROPE = 0, PAIR_SILU = 1 };
// The register-tiled Q8 product for many rows of x (q8_gemm.cu), same arguments and modes as
// q8_linear_launch; k a multiple of 32, x and wq 16-byte aligned.
int q8_gemm_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias, size_t n,
                   int mode, float* out, int sm_count, cudaStream_t st);
// out[m][n_ff] = silu(x . Wg^T + bg) * (x . Wu^T + bu) on the same tiles (biases may be null).
int q8_gemm_silu_launch(const float* x, size_t m, size_t k, const int8_t* wg, const float* sg, const float* bg,
                        const int8_t* wu, const float* su, const float* bu, size_t n_ff, float* out, int sm_count,
                        cudaStream_t st);
// The same products on the tcgen05 tensor cores (q8_tc.cu) for m >= 16 and k a multiple of
// 64 (wu/su/bu non-null: the SiLU pair). Returns 1 when the shape is not covered (the caller
// runs the register-tiled kernel), 0 after a launch, -1 on a launch failure.
int q8_tc_launch(const float* x, size_t m, size_t k, const int8_t* wq, const float* ws, const float* bias, size_t n,
                 int mode, const int8_t* wu, const float* su, const float* bu, float* out, int sm_count,
                 cudaStream_t st);
struct PairParams;
// The RoPE pair and the Whisper decoder's q/k/v product on the tcgen05 kernel (q8_tc.cu),
// for 16+ rows with k a multiple of 64 and every matrix's rows a multiple of 128; same
// return convention as q8_tc_launch.
int q8_tc_rope_launch(const PairParams& p, int sm_count, cudaStream_t st);
int q8_tc_qkv_launch(const PairParams& p, int sm_count, cudaStream_t st);
// The RoPE pair of q8_pair_launch on the same tiles.
int q8_gemm_rope_launch(const PairParams& p, int sm_count, cudaStream_t st);
// The Whisper decoder's q/k/v projections as one tiled product (16+ rows of x): q to
// p.q_out, k and v appended to the decoder caches p.cache_kt / p.cache_v (window w at
// w * p.cache_bs, row n_past + t of p.n_tok, p.d = n_state).
int q8_gemm_qkv_launch(const PairParams& p, int sm_count, cudaStream_t st);
struct PairParams {
    const float* x;  // [m][k], row t of the call is sequence t / n_tok, token t % n_tok
    int m, k;
    int m0;          // row of the call x[0] is (the launcher walks m in chunks)
    const int8_t* wq[3];
    const float* ws[3];
    const float* bias[3];  // per matrix, may be null
    int n_pairs;           // ROPE: (n_head + 2 n_head_kv) * d / 2; SILU: n_ff
    // ROPE
    int n_head, n_head_kv, d, n_tok, n_past, n_ctx;
    const float* cos_tab;
    const float* sin_tab;
    float* q_out;     // [m][n_head * d]
    float* cache_kt;  // sequence s at s * cache_bs: [n_head_kv][d][n_ctx]
    float* cache_v;   // sequence s at s * cache_bs: [n_ctx][n_head_kv * d]
    size_t cache_bs;
    // SILU
    float* out;  // [m][n_ff]
};
int q8_pair_launch(const PairParams& p, int epi, cudaStream_t st);

// Decode-step kernels around the projections (llm_step.cu), chained launches.
int rms_norm_launch(const float* x, size_t x_stride, size_t m, size_t n, const float* w, float eps, float* out,
                    size_t out_stride, cudaStream_t st);
int layer_norm_launch(const float* x, size_t x_stride, size_t m, size_t n, const float* w, const float* b, float eps,
                      float* out, size_t out_stride, cudaStream_t st);
// rows of the Q8 table for each token; with pe, row i also adds pe[(pos0 + i % n_tok) * k ..]
int embed_q8_launch(const int32_t* tokens, size_t m, const int8_t* q, const float* scales, size_t n_vocab,
                    size_t k, const float* pe, size_t pos0, size_t n_tok, float* out, int* err, cudaStream_t st);
int greedy_launch(float* logits, size_t m, size_t n_vocab, const int32_t* recent, size_t recent_stride,
                  size_t n_recent, size_t window, float penalty, int32_t* out, size_t out_stride, int* err,
                  cudaStream_t st);

// One bounded wait that nothing completes (selftest.cu); gave_up is set to 1 when it ran out.
int wait_timeout_selftest_launch(int* err, int* gave_up, cudaStream_t st);

// Elementwise helpers (misc.cu).
int f32_to_bf16_launch(const float* x, uint16_t* y, size_t n, cudaStream_t st);

struct RopeParams {
    float* q;
    const float* k;
    const float* v;
    float* cache_kt;
    float* cache_v;
    const float* cos_tab;
    const float* sin_tab;
    size_t n, n_past, n_head, n_head_kv, d, n_ctx;
    size_t q_bs, kv_bs, cache_bs;
};
int rope_kt_append_launch(const RopeParams& p, size_t n_batch, cudaStream_t st);

}  // namespace zwg
