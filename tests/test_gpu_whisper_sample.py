"""Whisper's greedy decoding rules on the device (include/zwgpu.h: zwg_whisper_sample,
zwg_whisper_step, zwg_whisper_decode_q8) against the oracle (oracle/transcribe.py), whose
rules and window loop reproduce the reference binary's transcription
(tests/test_transcribe_oracle.py).

Parity is exact for token ids and timestamps: every crafted logit row of
tests/whisper_sample_cases.py (one per rule branch, plus seeded random rows) must give the
oracle's (id, tid) and leave the logits row bit-identical to the oracle's (suppressions and
hotword additions are exact). The window loop's bookkeeping runs on the device over random
logits for several windows and must end every window as the oracle's loop does. The whole
window loop on the device (Q8 decoder + sampler, tokens fed back on the device) must give
the oracle's token stream for two windows of the seeded synthetic tiny.en model; the
oracle decoder uses the same Q8 weights (the current source's decoder, src/decoder.zig:
220-229; the binary's older build keeps f16 weights, which the oracle's f16 mode pins).
"""
import numpy as np
import pytest

from oracle import q8
from oracle import transcribe as T
from oracle import whisper as W
from tests.conftest import has_gpu
from tests.whisper_sample_cases import BEG, N_VOCAB, TOK, cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    ops.set_math("f32")
    return torch, ops


def _i32(torch, xs):
    return torch.tensor(xs, dtype=torch.int32, device="cuda:0")


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_sample_matches_oracle(env, case):
    torch, ops = env
    rules = ops.WhisperRules(hotwords=case["hotwords"])
    lg = case["logits"]
    dl = torch.from_numpy(lg.copy()).to("cuda:0").view(1, -1)
    cur = case["cur"]
    tokens = _i32(torch, [cur if cur else [0]])
    ids, tids = ops.whisper_sample(dl, tokens, _i32(torch, [len(cur)]), _i32(torch, [int(case["has_ts"])]),
                                   _i32(torch, [case["seek_delta"]]), rules)
    want_lg = lg.copy()
    want = T.sample(want_lg, cur, case["is_initial"], case["has_ts"], case["seek_delta"],
                    T.Rules(hotwords=case["hotwords"]))
    assert (int(ids.item()), int(tids.item())) == want
    got_lg = dl.cpu().numpy()[0]
    assert np.array_equal(got_lg, want_lg), "the logits row differs from the oracle's after the rules"


def test_sample_batched_rows(env):
    """All crafted rows without hotwords in one call: each row has its own window state."""
    torch, ops = env
    cs = [c for c in cases() if not c["hotwords"]]
    cap = max(1, max(len(c["cur"]) for c in cs))
    lg = np.stack([c["logits"] for c in cs])
    tok = np.zeros((len(cs), cap), np.int32)
    for i, c in enumerate(cs):
        tok[i, :len(c["cur"])] = c["cur"]
    dl = torch.from_numpy(lg.copy()).to("cuda:0")
    ids, tids = ops.whisper_sample(dl, torch.from_numpy(tok).to("cuda:0"), _i32(torch, [len(c["cur"]) for c in cs]),
                                   _i32(torch, [int(c["has_ts"]) for c in cs]), _i32(torch, [c["seek_delta"] for c in cs]))
    for i, c in enumerate(cs):
        want = T.sample(c["logits"].copy(), c["cur"], c["is_initial"], c["has_ts"], c["seek_delta"], T.Rules())
        assert (int(ids[i]), int(tids[i])) == want, c["name"]


def test_step_bookkeeping_matches_oracle_loop(env):
    """zwg_whisper_step over 80 steps of seeded random logits for six windows with different
    seek / seek_end (far from and near the end of the audio) and an n_max of 60: the tokens,
    timestamps, result lengths, seek deltas and failures equal the oracle loop's."""
    torch, ops = env
    from zwhisper_b200 import _lib
    import ctypes
    rng = np.random.default_rng(5)
    nb, cap, n_max = 6, 64, 60
    seeks = [0, 0, 3000, 6000, 0, 9000]
    ends = [10 ** 6, 2900, 5500, 10 ** 6, 4000, 9500]
    rules = ops.WhisperRules()
    win = torch.zeros(nb, 8, dtype=torch.int32, device="cuda:0")
    win[:, 0] = torch.tensor(seeks, dtype=torch.int32)
    win[:, 1] = torch.tensor(ends, dtype=torch.int32)
    tokens = torch.full((nb, cap), -1, dtype=torch.int32, device="cuda:0")
    tids = torch.full((nb, cap), -1, dtype=torch.int32, device="cuda:0")
    nxt = torch.zeros(nb, dtype=torch.int32, device="cuda:0")
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.zwg_whisper_window_init(win.data_ptr(), nb, ctypes.byref(rules.c), stream))
    states = [T.new_window_state(1500) for _ in range(nb)]
    done = [False] * nb
    for i in range(80):
        lg = (rng.standard_normal((nb, N_VOCAB)) * 2).astype(np.float32)
        # timestamps that move forward most of the time, text in between
        for b in range(nb):
            lg[b, BEG:] -= np.float32(rng.uniform(0.0, 6.0))
            lg[b, BEG + min(1500, 2 + 3 * i)] += np.float32(rng.uniform(0.0, 12.0))
            if rng.uniform() < 0.05:
                lg[b, TOK.eot] += 20.0
        dl = torch.from_numpy(lg.copy()).to("cuda:0")
        _lib.check(lib.zwg_whisper_step(dl.data_ptr(), nb, N_VOCAB, win.data_ptr(), tokens.data_ptr(), tids.data_ptr(),
                                        cap, ctypes.byref(rules.c), n_max, nxt.data_ptr(), stream))
        for b in range(nb):
            st = states[b]
            if done[b] or len(st["tokens"]) >= n_max:
                done[b] = True
                continue
            k = len(st["tokens"])
            s_id, s_tid = T.sample(lg[b].copy(), st["tokens"], k == 0, st["has_ts"], st["seek_delta"], T.Rules())
            done[b] = T.window_step(st, s_id, s_tid, k, n_max, seeks[b], ends[b], TOK, 3000) or k + 1 >= n_max
    w = win.cpu().numpy()
    tk, td = tokens.cpu().numpy(), tids.cpu().numpy()
    for b in range(nb):
        st = states[b]
        n = int(w[b, 2])
        assert tk[b, :n].tolist() == st["tokens"], f"window {b}"
        assert td[b, :n].tolist() == st["tids"], f"window {b}"
        assert (int(w[b, 3]), bool(w[b, 4]), int(w[b, 5]), bool(w[b, 6]), bool(w[b, 7])) == \
            (st["seek_delta"], st["has_ts"], st["result_len"], st["failed"], done[b]), f"window {b}"


def _oracle_q8_decoder(Wd, hp):
    dec = W.Decoder(Wd, hp, weights="q8")
    for name in list(dec.q8):
        qq, ss = q8.quantize(Wd[name].astype(np.float32))
        dec.q8[name] = q8.dequant(qq, ss)
    return dec


def test_decode_window_matches_oracle(env):
    """Two windows of the seeded synthetic tiny.en model decoded together on the device
    (zwg_whisper_decode_q8: prompt [sot], Q8 decoder steps and the sampler, tokens fed back on
    the device, the host reading only the windows' states): the 30 s clip from its start
    and the 95 s clip from frame 2968 (its second window), each against the oracle's loop
    over the same encoder output."""
    torch, ops = env
    hp = W.TINY_EN
    Wd = W.weights_dict(W.synth_model(hp, seed=0))
    wins = []
    for secs, seek in ((30.0, 0), (95.0, 2968)):
        pcm = W.synth_audio(secs, seed=0)
        mel = W.log_mel(W.pcm_to_f32(pcm), W.mel_filters(80))
        wins.append((W.encode(Wd, hp, mel, seek), seek, 1 + (len(pcm) + 200 - 400) // 160))
    Wg = ops.DecoderWeightsQ8(Wd, hp.n_text_layer)
    st = ops.DecoderState(hp.n_text_layer, len(wins), hp.n_text_state, hp.n_text_head, hp.n_text_ctx, hp.n_audio_ctx)
    for b, (enc, _, _) in enumerate(wins):
        st.set_audio_q8(Wg, b, torch.from_numpy(enc).to("cuda:0"))
    prompt = _i32(torch, [[TOK.sot]] * len(wins))
    got = ops.whisper_decode_q8(st, Wg, prompt, [w[1] for w in wins], [w[2] for w in wins], check_every=8)
    st.close()
    for b, (enc, seek, seek_end) in enumerate(wins):
        dec = _oracle_q8_decoder(Wd, hp)
        dec.set_audio(enc)
        want = T.decode_window(dec.forward, [TOK.sot], seek, seek_end, T.Rules(), hp.n_text_ctx)
        g = got[b]
        assert g["tokens"] == want.tokens, f"window {b}: first difference at " \
            f"{next(i for i, (x, y) in enumerate(zip(g['tokens'], want.tokens + [None] * 999)) if x != y)}"
        assert g["tids"] == want.tids
        assert (g["result_len"], g["seek_delta"], g["has_ts"], g["failed"]) == \
            (want.result_len, want.seek_delta, want.has_ts, want.failed)
