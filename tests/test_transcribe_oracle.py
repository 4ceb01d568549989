"""The oracle's restatement of the reference's greedy long-form decoding (oracle/transcribe.py),
pinned on the CPU:
  - every crafted logit row of tests/whisper_sample_cases.py gives the (id, tid) its rules
    imply, worked out by hand (src/transcribe.zig:491-580);
  - the window bookkeeping ends and fails windows as src/transcribe.zig:319-364 does;
  - the whole transcription of the synthetic tiny.en model reproduces every segment (start,
    end, token ids, text) that the reference's own binary printed for the same seeded model
    and audio (tests/golden/make_golden_transcribe.py): 30 s without the previous-window
    prompt, and 95 s (four windows) with it. The decoder runs with the binary's f16 weights
    (oracle.whisper.Decoder(weights="f16")).
"""
import json
import os

import numpy as np
import pytest

from oracle import transcribe as T
from oracle import whisper as W
from tests.whisper_sample_cases import BEG, TOK, cases

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "whisper_tiny_transcribe.json")


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_sample_rules(case):
    rules = T.Rules(hotwords=case["hotwords"])
    lg = case["logits"].copy()
    s_id, s_tid = T.sample(lg, case["cur"], case["is_initial"], case["has_ts"], case["seek_delta"], rules)
    assert TOK.beg <= s_tid < lg.size
    if case["expect"] is not None:
        want_id, want_tid = case["expect"]
        assert s_id == want_id
        if want_tid is not None:
            assert s_tid == want_tid


def test_initial_timestamp_limit():
    assert T.initial_ts_limit(T.Rules()) == 50          # 1 s at 20 ms per step
    assert T.initial_ts_limit(T.Rules(max_initial_ts=0.5)) == 25


def test_window_bookkeeping():
    tok, window = TOK, 3000

    def run(ids, seek=0, seek_end=10 ** 6, n_max=220):
        st = T.new_window_state(1500)
        for i, x in enumerate(ids):
            if T.window_step(st, x, BEG, i, n_max, seek, seek_end, tok, window):
                return st, i
        return st, None

    # text, timestamp, text, timestamp: result through the last timestamp
    st, end = run([100, BEG + 10, BEG + 10, 200, BEG + 30, tok.eot])
    assert end == 5 and not st["failed"] and st["result_len"] == 5 and st["seek_delta"] == 60
    # a timestamp that goes backwards after more text fails the window
    st, end = run([100, BEG + 30, 200, 300, BEG + 20])
    assert st["failed"] and end == 4 and st["result_len"] == 2
    # eot before any timestamp, far from the end of the audio: failed with nothing usable
    st, end = run([100, 200, tok.eot])
    assert st["failed"] and st["result_len"] == 0
    # ... but near the end of the audio the whole window is used
    st, end = run([100, 200, tok.eot], seek=0, seek_end=2900)
    assert not st["failed"] and st["result_len"] == 3
    # n_max tokens without a timestamp: failed
    st, end = run([100] * 5, n_max=5)
    assert st["failed"] and end == 4


@pytest.mark.parametrize("name", ["30s_no_context", "95s_context"])
def test_transcription_matches_reference_binary(name):
    with open(GOLDEN) as f:
        g = json.load(f)
    case = next(c for c in g["cases"] if c["name"] == name)
    hp = W.TINY_EN
    Wd = W.weights_dict(W.synth_model(hp, seed=g["model_seed"]))
    pcm = W.synth_audio(case["seconds"], seed=g["audio_seed"])
    mel = W.log_mel(W.pcm_to_f32(pcm), W.mel_filters(80))
    n_len_org = 1 + (len(pcm) + 200 - 400) // 160      # mel.zig:118
    dec = W.Decoder(Wd, hp, weights="f16")

    def encode_window(seek):
        dec.set_audio(W.encode(Wd, hp, mel, seek))

    def reset():
        dec.n_past = 0

    segs, _ = T.transcribe(encode_window, dec.forward, reset, n_len_org, T.Rules(), T.synthetic_text,
                           condition_on_previous=case["context"])
    want = case["segments"]
    assert len(segs) == len(want)
    for a, b in zip(segs, want):
        assert (a["t0"], a["t1"], a["tokens"], a["text"]) == (b["t0"], b["t1"], b["tokens"], b["text"])
