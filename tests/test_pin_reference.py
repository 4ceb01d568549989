"""Pin of the oracle against outputs of the reference itself (CPU, no GPU).

The fixture holds the shipped reference binary's `mel` and `logits` outputs for a seeded
synthetic tiny.en model and 30 s of seeded synthetic audio (tests/golden/make_golden.py).
The logits come from the whole encoder (4 layers of 6-head attention over 1500 frames)
and one decoder step (self- and cross-attention in 4 layers), so agreement at ~1e-6
pins the attention restatement together with everything around it.
"""
import numpy as np

from oracle import whisper as W
from tests.whisper_case import golden, logits_error, tiny_case


def test_mel_matches_reference_binary():
    g = golden()
    _, _, mel = tiny_case()
    assert tuple(mel.shape) == tuple(g["mel_shape"])
    np.testing.assert_allclose(mel[:, g["mel_frames"]], g["mel_sample"], atol=1e-4, rtol=0)


def test_forward_logits_match_reference_binary():
    """The binary is an older build whose decoder keeps f16 weights (no Q8); with the same
    weights the oracle's logits agree with it to ~1e-6."""
    g = golden()
    hp, Wd, mel = tiny_case()
    enc = W.encode(Wd, hp, mel, 0)
    dec = W.Decoder(Wd, hp, weights="f16")
    dec.set_audio(enc)
    logits = dec.forward([W.SOT])
    assert logits.size == int(g["n_vocab"])
    assert int(logits.argmax()) == int(g["argmax"])
    assert logits_error(logits) < 1e-4
    np.testing.assert_allclose(logits[g["logits_top_idx"]], g["logits_top"], atol=1e-4, rtol=0)
    assert abs(logits.astype(np.float64).sum() - float(g["logits_sum"])) < 1e-2
    # the current source's Q8 decoder (src/decoder.zig:220-229) keeps the greedy token
    dq = W.Decoder(Wd, hp, weights="q8")
    dq.set_audio(enc)
    assert int(dq.forward([W.SOT]).argmax()) == int(g["argmax"])
