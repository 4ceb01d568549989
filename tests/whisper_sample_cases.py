"""Crafted logit rows for Engine.sample (src/transcribe.zig:491-580), one per branch of its
rules, plus seeded random rows. Shared by the CPU tests of the oracle and the GPU parity
tests of the device sampler. Each case: logits (f32 [n_vocab]), the window's tokens so
far, is_initial, has_ts, seek_delta, and `expect` = the (id, tid) worked out by hand from
the rules (None where only the oracle decides)."""
import numpy as np

from oracle import transcribe as T

N_VOCAB = 51864
TOK = T.Tokens()
BEG = TOK.beg


def _base(seed, ts_offset=-5.0):
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal(N_VOCAB).astype(np.float32)
    lg[BEG:] += np.float32(ts_offset)
    return lg


def cases():
    out = []

    def add(name, lg, cur, is_initial, has_ts, seek_delta, expect=None, hotwords=()):
        out.append({"name": name, "logits": lg.astype(np.float32), "cur": list(cur), "is_initial": is_initial,
                    "has_ts": has_ts, "seek_delta": seek_delta, "expect": expect, "hotwords": [list(h) for h in hotwords]})

    # 1. first token, text wins; eot and " " are suppressed even when largest
    lg = _base(1)
    lg[TOK.eot] = 50.0
    lg[TOK.space] = 40.0
    lg[1234] = 30.0
    add("initial_text_wins", lg, [], True, False, 3000, (1234, None))
    # 2. first token, the timestamp block's total beats the best text token: 51 allowed
    # timestamps at 3.0 sum to 3 + log(51) = 6.93 > 4; later timestamps are cut by
    # max_initial_ts (1 s = 50 steps) even when larger
    lg = np.full(N_VOCAB, -30.0, np.float32)
    lg[:BEG] = np.float32(-5.0)
    lg[777] = 4.0
    lg[BEG:BEG + 51] = 3.0
    lg[BEG + 51:] = 10.0
    add("initial_timestamp_block_wins", lg, [], True, False, 3000, (BEG, BEG))
    # 3. the same block at 1.0 (1 + log 51 = 4.93) loses to a text token at 5.0
    lg[BEG:BEG + 51] = 1.0
    lg[777] = 5.0
    add("initial_text_beats_block", lg, [], True, False, 3000, (777, BEG))
    # 4. after text then a timestamp: text is suppressed, eot or a timestamp follows
    lg = _base(4)
    lg[TOK.eot] = 9.0
    lg[500] = 20.0
    add("pair_open_after_text", lg, [500, BEG + 10], False, True, 20, (TOK.eot, None))
    # 5. after two timestamps: timestamps are suppressed, text follows
    lg = _base(5, ts_offset=+20.0)
    lg[4321] = 15.0
    add("pair_closed", lg, [BEG + 5, BEG + 10], False, True, 20, (4321, BEG))
    # 6. timestamps before seek_delta / 2 steps are suppressed; the best allowed one wins
    lg = np.full(N_VOCAB, -20.0, np.float32)
    lg[BEG + 5] = 9.0
    lg[BEG + 25] = 8.0
    lg[BEG + 40] = 7.5
    add("seek_delta_bound", lg, [300], False, True, 50, (BEG + 25, BEG + 25))
    # 7. special tokens are always suppressed
    lg = _base(7)
    for t in (TOK.not_, TOK.sot, TOK.nosp, TOK.solm, TOK.translate, TOK.transcribe, TOK.prev):
        lg[t] = 100.0
    lg[42] = 50.0
    add("specials_suppressed", lg, [10, 11], False, False, 3000, (42, None))
    # 8. a hotword continuation gets the bias (5.0) and wins; a form with no matched prefix
    # gets half the bias on its first token
    lg = _base(8)
    lg[700] = 6.0
    lg[701] = 8.0
    lg[800] = 5.0
    add("hotword_continuation", lg, [12, 500, 600], False, False, 3000, (700, None),
        hotwords=[[500, 600, 700, 710], [800, 900]])
    lg = _base(9)
    lg[800] = 6.0
    lg[801] = 8.0
    add("hotword_first_token", lg, [12, 13], False, False, 3000, (800, None), hotwords=[[800, 900]])
    # 9. ties: the first index of the largest value wins
    lg = np.full(N_VOCAB, -3.0, np.float32)
    lg[BEG:] = -30.0
    lg[100] = 2.0
    lg[200] = 2.0
    add("tie_first_index", lg, [5], False, False, 3000, (100, BEG))
    # 10. everything suppressed but the specials and eot: eot wins
    lg = np.full(N_VOCAB, -np.inf, np.float32)
    lg[TOK.eot] = -1.0
    add("only_eot", lg, [5], False, False, 3000, (TOK.eot, BEG))
    # 11. seeded random rows with random window states
    rng = np.random.default_rng(11)
    for i in range(24):
        lg = (rng.standard_normal(N_VOCAB) * rng.uniform(0.5, 4.0)).astype(np.float32)
        lg[BEG:] += np.float32(rng.uniform(-3.0, 3.0))
        n_cur = int(rng.integers(0, 6))
        cur = [int(rng.choice([rng.integers(0, TOK.eot), rng.integers(BEG, N_VOCAB)])) for _ in range(n_cur)]
        has_ts = any(c > BEG for c in cur)
        seek_delta = int(rng.integers(0, 1500)) * 2 if has_ts else 3000
        hw = [[int(x) for x in rng.integers(0, 2000, size=int(rng.integers(1, 4)))] for _ in range(int(rng.integers(0, 3)))]
        add(f"random_{i}", lg, cur, n_cur == 0, has_ts, seek_delta, None, hotwords=hw)
    return out
