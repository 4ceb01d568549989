"""The synthetic tiny.en case the golden fixture pins (tests/golden/make_golden.py):
seeded model and audio rebuilt here, never read from the reference tree."""
import functools
import os

import numpy as np

from oracle import whisper as W

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "whisper_tiny_synth.npz")


@functools.lru_cache(maxsize=1)
def golden():
    return dict(np.load(GOLDEN))


@functools.lru_cache(maxsize=1)
def tiny_case():
    g = golden()
    model_seed, audio_seed = (int(x) for x in g["seeds"])
    hp = W.TINY_EN
    tensors = W.synth_model(hp, seed=model_seed)
    filters = W.mel_filters(80)
    pcm = W.synth_audio(30.0, seed=audio_seed)
    mel = W.log_mel(W.pcm_to_f32(pcm), filters)
    return hp, W.weights_dict(tensors), mel


def logits_error(logits: np.ndarray) -> float:
    g = golden()
    return float(np.abs(logits[g["logits_idx"]] - g["logits_sample"]).max())
