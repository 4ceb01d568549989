"""The whole Whisper front of a transcription on the device against the reference binary's
own output for the seeded synthetic tiny.en case (tests/golden, tests/whisper_case.py):
16 kHz samples -> log-mel (zwg_log_mel) -> encoder (zwg_enc_forward_f16: f16 tcgen05 GEMMs,
bf16 attention) -> one decoder step after [sot], once by the oracle decoder on the device
encoder's output and once entirely on the device (zwg_dec_set_audio_q8 + zwg_dec_forward_q8,
Q8 weights as the current source loads them, src/decoder.zig:220-229).

The device encoder rounds activations to f16 and attention operands to bf16 where the
reference computes in f32: measured on B200, the ln_post output is within 7.3e-4 of the
oracle encoder's and the binary's top logits within 2.2e-5; the bounds below keep 7x and
20x of that, and the greedy token must be the binary's."""
import numpy as np
import pytest

from oracle import whisper as W
from tests.conftest import has_gpu
from tests.whisper_case import golden, tiny_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    ops.set_math("f32")
    return torch, ops


def test_audio_to_logits_on_device(env):
    torch, ops = env
    g = golden()
    hp, Wd, mel_o = tiny_case()
    _, audio_seed = (int(x) for x in g["seeds"])
    samples = W.pcm_to_f32(W.synth_audio(30.0, seed=audio_seed))
    filters = W.mel_filters(hp.n_mels)
    dev = torch.device("cuda:0")
    mel_d = ops.log_mel(torch.from_numpy(samples).to(dev), torch.from_numpy(filters).to(dev))
    assert np.abs(mel_d.cpu().numpy() - mel_o).max() < 1e-4
    Wg = ops.EncoderWeightsF16(Wd, hp.n_audio_layer, hp.n_audio_head)
    enc = ops.encoder_forward(Wg, mel_d, 1)
    enc_o = W.encode(Wd, hp, mel_o, 0)
    enc_err = float(np.abs(enc.cpu().numpy()[0] - enc_o).max())

    # the oracle decoder (f16 weights, as the binary) on the device encoder's output
    dec = W.Decoder(Wd, hp, weights="f16")
    dec.set_audio(enc.cpu().numpy()[0])
    logits = dec.forward([W.SOT])
    top_err = float(np.abs(logits[g["logits_top_idx"]] - g["logits_top"]).max())
    print(f"encoder max err {enc_err:.3e}, top-logit err {top_err:.3e}")
    assert int(logits.argmax()) == int(g["argmax"])
    assert enc_err < 5e-3 and top_err < 5e-4

    # everything on the device: Q8 decoder weights, cross K/V from the device encoder
    Wq = ops.DecoderWeightsQ8(Wd, hp.n_text_layer)
    st = ops.DecoderState(hp.n_text_layer, 1, hp.n_text_state, hp.n_text_head, hp.n_text_ctx, hp.n_audio_ctx)
    st.set_audio_q8(Wq, 0, enc[0].contiguous())
    _, logits_d = st.forward_q8(Wq, torch.tensor([[W.SOT]], dtype=torch.int32, device=dev), 0)
    assert int(logits_d[0].argmax()) == int(g["argmax"])
    st.close()
