"""Where the device encoder's deviation from the oracle comes from (CPU, no GPU).

The device encoder (csrc/enc_api.cu) computes Encoder.forward (src/encoder.zig:118-179)
with the reference's f32 accumulation but rounds the operands it hands to the tensor cores:
the mel rows and every GEMM input to f16 (the LayerNorm outputs, the attention output, the
MLP hidden rows after GELU, conv1's output), q, k, v to bf16 and the probabilities P to bf16
inside the attention. This test restates the oracle encoder with exactly those roundings
(numpy, float32 otherwise) on the config-0 tiny.en case of the golden fixture and checks
that they alone move the ln_post output by the amount the GPU test observes for the device
(max 7.3e-4, tests/test_gpu_whisper_pipeline.py): the device tolerance is the rounding
budget of the f16/bf16 operands, not slack for an error elsewhere."""
import numpy as np

from oracle import whisper as W
from tests.whisper_case import tiny_case


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def bf16(x):
    """Round f32 to bf16 (to nearest even) and back."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def attention_bf16(q, k, v, n_head):
    """Non-causal attention with bf16 q, k, v and bf16 P against f32 row sums, f32 out."""
    n, ns = q.shape
    d = ns // n_head
    out = np.empty((n, ns), np.float32)
    q, k, v = bf16(q), bf16(k), bf16(v)
    for h in range(n_head):
        sl = slice(h * d, (h + 1) * d)
        s = (q[:, sl] @ k[:, sl].T) * np.float32(1.0 / np.sqrt(d))
        p = np.exp(s - s.max(1, keepdims=True)).astype(np.float32)
        out[:, sl] = (bf16(p) @ v[:, sl]) / p.sum(1, keepdims=True)
    return out


def encode_device_rounding(Wd, hp, mel):
    n_ctx, ns, H = hp.n_audio_ctx, hp.n_audio_state, hp.n_audio_head
    T = 2 * n_ctx
    melr = f16(mel)
    col = np.zeros((T, hp.n_mels, 3), np.float32)
    for kk in range(3):
        ti = np.arange(T) + kk - 1
        ok = (ti >= 0) & (ti < T) & (ti < mel.shape[1])
        col[ok, :, kk] = melr[:, ti[ok]].T
    w1 = f16(Wd["encoder.conv1.weight"].reshape(ns, -1))
    x = f16(W.gelu(W.linear(col.reshape(T, -1), w1, Wd["encoder.conv1.bias"])))
    col2 = np.zeros((n_ctx, ns, 3), np.float32)
    for kk in range(3):
        ti = 2 * np.arange(n_ctx) + kk - 1
        ok = (ti >= 0) & (ti < T)
        col2[ok, :, kk] = x[ti[ok]]
    w2 = f16(Wd["encoder.conv2.weight"].reshape(ns, -1))
    x = (W.gelu(W.linear(col2.reshape(n_ctx, -1), w2, Wd["encoder.conv2.bias"]))
         + Wd["encoder.positional_embedding"][:n_ctx]).astype(np.float32)
    for i in range(hp.n_audio_layer):
        p = f"encoder.blocks.{i}."
        h = f16(W.layer_norm(x, Wd[p + "attn_ln.weight"], Wd[p + "attn_ln.bias"]))
        q = W.linear(h, Wd[p + "attn.query.weight"], Wd[p + "attn.query.bias"])
        k = W.linear(h, Wd[p + "attn.key.weight"])
        v = W.linear(h, Wd[p + "attn.value.weight"], Wd[p + "attn.value.bias"])
        a = f16(attention_bf16(q, k, v, H))
        x = (x + W.linear(a, Wd[p + "attn.out.weight"], Wd[p + "attn.out.bias"])).astype(np.float32)
        h = f16(W.layer_norm(x, Wd[p + "mlp_ln.weight"], Wd[p + "mlp_ln.bias"]))
        h = f16(W.gelu(W.linear(h, Wd[p + "mlp.0.weight"], Wd[p + "mlp.0.bias"])))
        x = (x + W.linear(h, Wd[p + "mlp.2.weight"], Wd[p + "mlp.2.bias"])).astype(np.float32)
    return W.layer_norm(x, Wd["encoder.ln_post.weight"], Wd["encoder.ln_post.bias"])


def test_device_roundings_explain_the_encoder_tolerance():
    hp, Wd, mel = tiny_case()
    want = W.encode(Wd, hp, mel, 0)
    got = encode_device_rounding(Wd, hp, mel)
    err = float(np.abs(got - want).max())
    # measured 6.99e-4 here against the device's 7.3e-4 (tests/test_gpu_whisper_pipeline.py):
    # the bound holds the restatement to within about 2x of that figure
    assert 3e-4 < err < 1.5e-3, err
