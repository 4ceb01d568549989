"""The Whisper decoder step on the device (include/zwgpu.h: zwg_layer_norm, zwg_linear_q8_gelu,
zwg_dec_set_audio_q8, zwg_dec_forward_q8) against the oracle decoder (oracle/whisper.py,
src/decoder.zig:151-206), whose forward the golden fixture pins to the reference binary's
logits (tests/test_pin_reference.py).

Tolerances: LayerNorm to f32 rounding (rel 2e-6); GELU after a Q8 product to the product's
bound (relative 2e-6 of the sum of |terms|) plus tanh's; logits of whole decoder steps abs
1e-4 + rel 1e-4; the greedy tokens must be identical."""
import numpy as np
import pytest

from oracle import q8
from oracle import whisper as W
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    ops.set_math("f32")
    return torch, ops


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


@pytest.mark.parametrize("m,n", [(1, 384), (7, 512), (3, 1280)])
def test_layer_norm(env, m, n):
    torch, ops = env
    rng = np.random.default_rng(m + n)
    x = (rng.standard_normal((m, n), dtype=np.float32) * 3 + 1).astype(np.float32)
    w = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    got = ops.layer_norm(dev(torch, x), dev(torch, w), dev(torch, b)).cpu().numpy()
    np.testing.assert_allclose(got, W.layer_norm(x, w, b), rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("m", [1, 3, 37])
def test_linear_q8_gelu(env, m):
    torch, ops = env
    rng = np.random.default_rng(7 * m)
    n, k = 1536, 384
    x = rng.standard_normal((m, k), dtype=np.float32)
    qw, sw = q8.quantize((rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.05)).astype(np.float32))
    b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.5)).astype(np.float32)
    got = ops.linear_q8_gelu(dev(torch, x), dev(torch, qw), dev(torch, sw), dev(torch, b)).cpu().numpy()
    pre = q8.linear(x, qw, sw, b)
    want = W.gelu(pre)
    mag = np.abs(x).astype(np.float64) @ np.abs(q8.dequant(qw, sw)).astype(np.float64).T + np.abs(b)
    assert (np.abs(got - want) <= 2.2e-6 * mag + 2e-6 * np.abs(want) + 1e-7).all()


def small_hp():
    return W.Hparams(n_vocab=2000, n_audio_ctx=200, n_audio_state=128, n_audio_head=2, n_audio_layer=1,
                     n_text_ctx=64, n_text_state=128, n_text_head=2, n_text_layer=2)


def oracle_decoder(Wd, hp):
    """The oracle decoder with its Q8 matrices made by oracle/q8.py (the exact Q8.quantize
    rule, which the device quantizer reproduces bit for bit)."""
    dec = W.Decoder(Wd, hp, weights="q8")
    for name in list(dec.q8):
        qq, ss = q8.quantize(Wd[name].astype(np.float32))
        dec.q8[name] = q8.dequant(qq, ss)
    return dec


@pytest.mark.parametrize("B,q8_mode", [(1, 1), (3, 1), (16, 1), (16, "always")], ids=["1", "3", "16", "16-tcgen05"])
def test_decoder_forward_greedy(env, B, q8_mode):
    """A 3-token prompt for B windows with their own audio, then 4 greedy tokens fed back on
    the device (argmax without a penalty): logits within tolerance at every step, identical
    tokens. At 16 windows every projection runs a 16-row Q8 product and q/k/v one launch
    whose epilogue appends k and v to the caches: by default on the CUDA-core kernel (this
    model's matrices are small), with the switch at "always" on the tcgen05 kernel."""
    torch, ops = env
    prev = ops.q8_tensor_cores(q8_mode)
    try:
        run_decoder_forward_greedy(torch, ops, B)
    finally:
        ops.q8_tensor_cores(prev)


def run_decoder_forward_greedy(torch, ops, B):
    hp = small_hp()
    Wd = W.weights_dict(W.synth_model(hp, seed=21))
    rng = np.random.default_rng(22 + B)
    encs = [rng.standard_normal((hp.n_audio_ctx, hp.n_text_state), dtype=np.float32) for _ in range(B)]
    prompt = rng.integers(0, hp.n_vocab, (B, 3)).astype(np.int32)

    decs = [oracle_decoder(Wd, hp) for _ in range(B)]
    for d, e in zip(decs, encs):
        d.set_audio(e)

    Wg = ops.DecoderWeightsQ8(Wd, hp.n_text_layer)
    st = ops.DecoderState(hp.n_text_layer, B, hp.n_text_state, hp.n_text_head, hp.n_text_ctx, hp.n_audio_ctx)
    for w in range(B):
        st.set_audio_q8(Wg, w, dev(torch, encs[w]))
    # the cross K/V the device computed, against the oracle's (src/decoder.zig:154-155)
    for layer in range(hp.n_text_layer):
        _, _, ck, cv = st.cache_views(layer)
        for w in range(B):
            np.testing.assert_allclose(ck[w].cpu().numpy(), decs[w].cross_k[layer], atol=2e-5, rtol=1e-5)
            np.testing.assert_allclose(cv[w].cpu().numpy(), decs[w].cross_v[layer], atol=2e-5, rtol=1e-5)

    x, logits = st.forward_q8(Wg, dev(torch, prompt), 0)
    want = np.stack([d.forward(list(prompt[b])) for b, d in enumerate(decs)])
    np.testing.assert_allclose(logits.cpu().numpy(), want, atol=1e-4, rtol=1e-4)
    n_past = 3
    for step in range(4):
        tok = ops.llm_greedy(logits, penalty=1.0)
        got_t = tok.cpu().numpy().tolist()
        want_t = [int(np.argmax(want[b])) for b in range(B)]
        assert got_t == want_t, f"step {step}: {got_t} vs {want_t}"
        x, logits = st.forward_q8(Wg, tok.view(B, 1).contiguous(), n_past)
        want = np.stack([d.forward([want_t[b]]) for b, d in enumerate(decs)])
        np.testing.assert_allclose(logits.cpu().numpy(), want, atol=1e-4, rtol=1e-4)
        n_past += 1
    st.close()
