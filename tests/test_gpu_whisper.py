"""End-to-end parity on real attention inputs (config 0: tiny.en, one 30 s window).

1. The oracle's whisper forward with every attention call (4 encoder layers, 4 decoder
   self- and 4 cross-attention calls) routed through the GPU drop-in (zwg_attention):
   logits against the reference binary's own logits (tests/golden), identical argmax.
2. Per-layer encoder attention outputs [6][1500][64] of the bf16 tensor-core kernel
   against the f32 oracle, within the north-star tolerance (max-abs 2e-3, rel 1e-3).
"""
import numpy as np
import pytest

from oracle import attention as A
from oracle import whisper as W
from tests.conftest import has_gpu
from tests.whisper_case import golden, logits_error, tiny_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    from zwhisper_b200 import ops as o
    return o


def gpu_attention(ops):
    def fn(q, k, v, n_q, n_kv, n_state, n_head, causal):
        out = ops.attention(q.reshape(-1), k.reshape(-1), v.reshape(-1), n_q, n_kv, n_state, n_head, causal)
        return out.reshape(n_q, n_state)
    return fn


def test_tiny_forward_through_gpu_matches_reference_logits(ops):
    g = golden()
    hp, Wd, mel = tiny_case()
    att = gpu_attention(ops)
    enc = W.encode(Wd, hp, mel, 0, attention=att)
    dec = W.Decoder(Wd, hp, attention=att, weights="f16")
    dec.set_audio(enc)
    logits = dec.forward([W.SOT])
    assert int(logits.argmax()) == int(g["argmax"])
    assert logits_error(logits) < 1e-4


def test_encoder_layers_tensor_core_vs_oracle(ops):
    """Config 0 check: per-layer attention outputs of the tcgen05 kernel (bf16 operands,
    f32 softmax and accumulation) on the real Q/K/V of the synthetic window."""
    import torch
    hp, Wd, mel = tiny_case()
    rec = []
    W.encode(Wd, hp, mel, 0, record=rec)
    n_ctx, ns, H = hp.n_audio_ctx, hp.n_audio_state, hp.n_audio_head
    dev = torch.device("cuda:0")
    worst = 0.0
    for q, k, v, want in rec:
        tq, tk, tv = (ops.f32_to_bf16(torch.from_numpy(np.ascontiguousarray(x)).to(dev).view(1, n_ctx, ns))
                      for x in (q, k, v))
        got = ops.enc_attn_bf16(tq, tk, tv, H).cpu().numpy().reshape(n_ctx, ns)
        np.testing.assert_allclose(got, want, atol=2e-3, rtol=1e-3)
        worst = max(worst, float(np.abs(got - want).max()))
        # the f32 path on the same inputs holds the reference's unit-test tolerance
        got32 = ops.attention(q, k, v, n_ctx, n_ctx, ns, H, False).reshape(n_ctx, ns)
        np.testing.assert_allclose(got32, want, atol=1e-4, rtol=0)
    assert worst < 2e-3
