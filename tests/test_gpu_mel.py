"""Log-mel spectrogram on the device (csrc/mel.cu, zwg_log_mel) against the oracle's
restatement of mel.logMel (oracle/whisper.py log_mel, src/mel.zig:103-157).

Tolerance: the device sums each DFT bin in f32 in another order than the reference's radix-2
FFT (the oracle uses an f64 FFT); the mel sums and log10 run in f64 in all three. The power of
a bin differs by a few f32 roundings of the frame's largest terms, so the log10 of a mel sum
(then scaled by 1/4) differs by well under 1e-4, except where it sits at the clamp (max - 8),
which both sides reach exactly. The end-to-end check runs the device mel into the device
encoder and compares with the oracle encoder on the oracle mel."""
import numpy as np
import pytest

from oracle import whisper as W
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu

MEL_ATOL = 1e-4


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    return torch, ops


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


@pytest.mark.parametrize("seconds,seed", [(9.0, 1), (31.5, 2)])
def test_log_mel_matches_oracle(env, seconds, seed):
    torch, ops = env
    x = W.pcm_to_f32(W.synth_audio(seconds=seconds, seed=seed))
    filters = W.mel_filters(80)
    want = W.log_mel(x, filters)
    got = ops.log_mel(dev(torch, x), dev(torch, filters)).cpu().numpy()
    assert got.shape == want.shape
    err = np.abs(got - want)
    assert err.max() < MEL_ATOL, (float(err.max()), np.unravel_index(int(err.argmax()), err.shape))


def test_log_mel_short_and_silent(env):
    """250 samples (three real frames, the rest the floor; the reflection needs more than
    200 samples) and 2 s of silence (a flat spectrogram at the clamp floor, as the
    reference's own test expects)."""
    torch, ops = env
    filters = W.mel_filters(80)
    rng = np.random.default_rng(3)
    for x in (rng.standard_normal(250).astype(np.float32) * 0.1, np.zeros(32000, np.float32)):
        want = W.log_mel(x, filters)
        got = ops.log_mel(dev(torch, x), dev(torch, filters)).cpu().numpy()
        assert got.shape == want.shape
        assert np.abs(got - want).max() < MEL_ATOL
    assert np.all(got == got[0, 0])


def test_audio_to_encoder_on_device(env):
    """Samples -> device mel -> device encoder (2 consecutive windows) against the oracle
    encoder on the oracle mel, at the encoder tolerance of tests/test_gpu_encoder.py."""
    torch, ops = env
    hp = W.Hparams(n_vocab=2000, n_audio_ctx=256, n_audio_state=256, n_audio_head=4, n_audio_layer=1,
                   n_text_ctx=64, n_text_state=256, n_text_head=4, n_text_layer=1)
    Wd = W.weights_dict(W.synth_model(hp, seed=9, encoder_only=True))
    x = W.pcm_to_f32(W.synth_audio(seconds=6.0, seed=10))
    filters = W.mel_filters(hp.n_mels)
    mel = W.log_mel(x, filters)
    mel_d = ops.log_mel(dev(torch, x), dev(torch, filters))
    Wg = ops.EncoderWeightsF16(Wd, hp.n_audio_layer, hp.n_audio_head)
    got = ops.encoder_forward(Wg, mel_d, 2).cpu().numpy()
    T = 2 * hp.n_audio_ctx
    for b in range(2):
        want = W.encode(Wd, hp, mel, offset=b * T)
        err = np.abs(got[b] - want)
        assert err.max() < 3e-2 and err.mean() < 3e-3, (b, float(err.max()), float(err.mean()))
