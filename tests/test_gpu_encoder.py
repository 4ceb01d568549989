"""The Whisper encoder on the device: the f16 tcgen05 GEMM (csrc/gemm_tc.cu, zwg_gemm_f16)
against torch fp32 products of the same f16 operands, and the whole Encoder.forward
(csrc/enc_api.cu, zwg_enc_forward_f16) against the oracle encoder (oracle/whisper.py encode,
src/encoder.zig:118-179), whose forward the golden fixture pins to the reference binary.

Tolerances. GEMM: the f16 operands multiply exactly and accumulate in f32, so the result
differs from an fp32 sum of the same products only by the summation order: within 1e-5 of
the sum of |terms|; f16 / bf16 outputs add one rounding of their type. Encoder: the device
rounds activations to f16 before each product (relative 2^-11), q, k, v to bf16 (2^-8) for
the attention and P to bf16 inside it, while the oracle keeps f32 throughout; over the
blocks these roundings leave the ln_post output (values of order 1) within 3e-2 of the
oracle, 3e-3 on average, and the decoder's greedy token on that output must be the same."""
import numpy as np
import pytest

from oracle import whisper as W
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    return torch, ops


def ref_gemm(torch, a, w, bias, gelu, addend):
    y = a.float() @ w.float().T
    mag = a.float().abs() @ w.float().abs().T
    if bias is not None:
        y = y + bias
    if gelu:
        c = 0.7978845608028654
        y = 0.5 * y * (1.0 + torch.tanh(c * (y + 0.044715 * y * y * y)))
    if addend is not None:
        y = y + addend
    return y, mag


@pytest.mark.parametrize("B,M,N,K,out_dtype,gelu,acc,add", [
    (2, 1500, 384, 384, "f32", False, False, False),   # N tail of a 256-column tile
    (1, 3000, 768, 240, "f16", True, False, False),    # conv1-shaped: K tail of a 64-wide step
    (2, 1500, 2304, 768, "bf16", False, False, False),  # fused q/k/v projection
    (2, 700, 768, 3072, "f32", False, True, False),    # MLP down-projection into the residual
    (1, 1500, 768, 2304, "f32", True, False, True),    # conv2 + positional embedding
])
def test_gemm_f16(env, B, M, N, K, out_dtype, gelu, acc, add):
    torch, ops = env
    g = torch.Generator(device="cuda:0")
    g.manual_seed(B * M + N + K)
    a = (torch.randn(B, M, K, generator=g, device="cuda:0")).half()
    w = (torch.randn(N, K, generator=g, device="cuda:0") * 0.02).half()
    bias = torch.randn(N, generator=g, device="cuda:0") * 0.1
    addend = torch.randn(M, N, generator=g, device="cuda:0") if add else None
    dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[out_dtype]
    base = torch.randn(B, M, N, generator=g, device="cuda:0").to(dt) if acc else torch.zeros(B, M, N, device="cuda:0",
                                                                                               dtype=dt)
    out = base.clone()
    ops.gemm_f16(a, w, bias=bias, gelu=gelu, addend=addend, accumulate=acc, out=out, out_dtype=out_dtype)
    want, mag = ref_gemm(torch, a, w, bias, gelu, addend)
    if acc:
        want = want + base.float()
    got = out.float()
    ulp = {"f32": 0.0, "f16": 2.0 ** -10, "bf16": 2.0 ** -7}[out_dtype]
    bound = 1e-5 * (mag + bias.abs()) + ulp * want.abs() + 1e-6
    if gelu:
        bound = bound * 1.5 + 1e-6
    bad = (got - want).abs() > bound
    assert not bad.any(), f"{int(bad.sum())} elements off; max excess {float(((got - want).abs() - bound).max())}"


def test_gemm_overlapping_rows(env):
    """The convolutions' operand: row t of A is three consecutive rows of a [rows][C] buffer
    (lda = C, K = 3 C): the same product as an explicit im2col."""
    torch, ops = env
    g = torch.Generator(device="cuda:0")
    g.manual_seed(3)
    C, T, N = 80, 600, 256
    buf = torch.randn(2, T + 2, C, generator=g, device="cuda:0").half()
    w = (torch.randn(N, 3 * C, generator=g, device="cuda:0") * 0.05).half()
    out = torch.zeros(2, T, N, device="cuda:0")
    ops.gemm_f16(buf, w, out=out, M=T, K=3 * C, lda=C, a_bs=(T + 2) * C)
    col = torch.stack([buf[:, t:t + 3].reshape(2, -1) for t in range(T)], dim=1)
    want = col.float() @ w.float().T
    mag = col.float().abs() @ w.float().abs().T
    assert ((out - want).abs() <= 1e-5 * mag + 1e-6).all()


def small_hp(n_layer=2):
    return W.Hparams(n_vocab=2000, n_audio_ctx=256, n_audio_state=256, n_audio_head=4, n_audio_layer=n_layer,
                     n_text_ctx=64, n_text_state=256, n_text_head=4, n_text_layer=2)


def test_encoder_forward_matches_oracle(env):
    """Two windows of synthetic speech-like audio (the second one runs past the end of the
    mel, so its tail frames are zero) through a 2-block encoder; then one decoder step on
    each window's output must give the oracle's greedy token."""
    torch, ops = env
    hp = small_hp()
    tensors = W.synth_model(hp, seed=5)
    Wd = W.weights_dict(tensors)
    samples = W.pcm_to_f32(W.synth_audio(seconds=9.0, seed=4))
    mel = W.log_mel(samples, W.mel_filters(hp.n_mels))
    T = 2 * hp.n_audio_ctx
    offsets = [0, mel.shape[1] - T // 2]
    want = np.stack([W.encode(Wd, hp, mel, offset=o) for o in offsets])

    Wg = ops.EncoderWeightsF16(Wd, hp.n_audio_layer, hp.n_audio_head)
    mel_d = torch.from_numpy(np.ascontiguousarray(mel)).to("cuda:0")
    off_d = torch.tensor(offsets, dtype=torch.int32, device="cuda:0")
    got = ops.encoder_forward(Wg, mel_d, len(offsets), offsets=off_d).cpu().numpy()
    err = np.abs(got - want)
    assert err.max() < 3e-2 and err.mean() < 3e-3, (float(err.max()), float(err.mean()))

    # the decoder's greedy token after [sot] on either encoder output
    for b in range(len(offsets)):
        toks = []
        for enc in (want[b], got[b]):
            dec = W.Decoder(Wd, hp)
            dec.set_audio(enc.astype(np.float32))
            toks.append(int(np.argmax(dec.forward([1]))))
        assert toks[0] == toks[1]


def test_encoder_consecutive_windows_default_offsets(env):
    """offsets NULL: window i starts at frame i * 2 n_ctx (consecutive 30 s windows)."""
    torch, ops = env
    hp = small_hp(n_layer=1)
    Wd = W.weights_dict(W.synth_model(hp, seed=6))
    samples = W.pcm_to_f32(W.synth_audio(seconds=12.0, seed=8))
    mel = W.log_mel(samples, W.mel_filters(hp.n_mels))
    T = 2 * hp.n_audio_ctx
    Wg = ops.EncoderWeightsF16(Wd, hp.n_audio_layer, hp.n_audio_head)
    mel_d = torch.from_numpy(np.ascontiguousarray(mel)).to("cuda:0")
    got = ops.encoder_forward(Wg, mel_d, 3).cpu().numpy()
    for b in range(3):
        want = W.encode(Wd, hp, mel, offset=b * T)
        err = np.abs(got[b] - want)
        assert err.max() < 3e-2 and err.mean() < 3e-3, (b, float(err.max()), float(err.mean()))
