"""CPU restatement of the reference's greedy long-form decoding rules (test infrastructure).

Follows src/transcribe.zig of the reference:
  - `sample`          Engine.sample (src/transcribe.zig:491-580): whisper.cpp's logit rules
                      (suppressed special tokens, timestamp pairing, the initial-timestamp
                      and seek-delta bounds), the hotword bias (applyHotwords,
                      src/transcribe.zig:176-193), the log-sum-exp of the timestamp block
                      against the best text token, then the argmax and the best timestamp.
  - `window_step`     the bookkeeping of one token in the window loop of Engine.transcribe
                      (src/transcribe.zig:319-364): seek_delta, has_ts, result_len and the
                      end and failure conditions.
  - `decode_window`   that loop for one window (src/transcribe.zig:292-365).
  - `window_segments` the segments the loop hands to its callback and the trailing text
                      segment after it (src/transcribe.zig:330-387, 457-489, without quote
                      splitting or voices), as the reference binary prints them with --json.
  - `transcribe`      the outer loop over windows (src/transcribe.zig:248-401): seek, the
                      prompt with the previous window's text, the skip of failed windows.

Only tests use this module; the GPU path never imports it. All arithmetic on logits is
f32 (numpy float32), as in the reference; the log-sum-exp sums run in numpy's order rather
than the reference's vector order, so a decision can differ only where the timestamp block
and the best text token tie to f32 rounding.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, List, Sequence, Tuple

import numpy as np

F32 = np.float32
NEG_INF = F32(-np.inf)


@dataclass(frozen=True)
class Tokens:
    """Special token ids of English-only models (src/model.zig:37-47); `space` is the id of
    the token " " (Engine.init: tokenId(" ") orelse 220, src/transcribe.zig:116)."""
    eot: int = 50256
    sot: int = 50257
    translate: int = 50357
    transcribe: int = 50358
    solm: int = 50359
    prev: int = 50360
    nosp: int = 50361
    not_: int = 50362
    beg: int = 50363
    space: int = 220


@dataclass
class Rules:
    """The inputs of Engine.sample besides the logits and the window's tokens."""
    tok: Tokens = field(default_factory=Tokens)
    n_audio_ctx: int = 1500
    max_initial_ts: float = 1.0                 # Options.max_initial_ts (src/transcribe.zig:42-43)
    hotwords: Sequence[Sequence[int]] = ()      # every form of every hotword, in order
    hotword_bias: float = 5.0                   # Engine.hotword_bias (src/transcribe.zig:94)


def initial_ts_limit(rules: Rules) -> int:
    """tid0 of the max_initial_ts rule (src/transcribe.zig:520-523): round(max / precision)
    in f32, precision = 30 / n_audio_ctx; @round rounds half away from zero."""
    precision = F32(30.0) / F32(rules.n_audio_ctx)
    q = F32(F32(rules.max_initial_ts) / precision)
    return int(np.floor(float(q) + 0.5))


def apply_hotwords(lg: np.ndarray, cur: Sequence[int], rules: Rules) -> None:
    """applyHotwords (src/transcribe.zig:176-193): for each form, the longest prefix of the
    form (shorter than the form) that matches the tail of `cur`; the form's next token, if
    it is text, gets the bias (half of it when the matched prefix is empty)."""
    eot = rules.tok.eot
    bias = F32(rules.hotword_bias)
    for form in rules.hotwords:
        if len(form) == 0:
            continue
        p = min(len(form) - 1, len(cur))
        while p > 0 and list(form[:p]) != list(cur[len(cur) - p:]):
            p -= 1
        nxt = form[p]
        if nxt < eot:
            lg[nxt] = F32(lg[nxt] + (bias * F32(0.5) if p == 0 else bias))


def sample(lg: np.ndarray, cur: Sequence[int], is_initial: bool, has_ts: bool, seek_delta: int,
           rules: Rules) -> Tuple[int, int]:
    """Engine.sample (src/transcribe.zig:491-580). `lg` (f32 logits) is modified in place, as
    the reference modifies Engine.logits. Returns (id, tid)."""
    assert lg.dtype == np.float32
    tok = rules.tok
    n = lg.shape[0]
    # src/transcribe.zig:498-509: special tokens
    if is_initial:
        lg[tok.eot] = NEG_INF
        lg[tok.space] = NEG_INF
    for t in (tok.not_, tok.sot, tok.nosp, tok.solm, tok.translate, tok.transcribe, tok.prev):
        lg[t] = NEG_INF
    # :511-519: timestamps come in pairs
    last_was_ts = len(cur) > 0 and cur[-1] >= tok.beg
    penultimate_was_ts = len(cur) < 2 or cur[-2] >= tok.beg
    if last_was_ts:
        if penultimate_was_ts:
            lg[tok.beg:] = NEG_INF
        else:
            lg[:tok.eot] = NEG_INF
    # :520-526: the first timestamp is at most max_initial_ts seconds
    if is_initial and rules.max_initial_ts > 0:
        tid0 = initial_ts_limit(rules)
        if tok.beg + tid0 + 1 < n:
            lg[tok.beg + tid0 + 1:] = NEG_INF
    # :527-530: timestamps never go backwards within the window
    if has_ts:
        tid0 = seek_delta // 2
        lg[tok.beg:tok.beg + tid0] = NEG_INF
    apply_hotwords(lg, cur, rules)

    # :532-545: log-probabilities (-inf entries contribute nothing)
    mx = lg.max()
    fin = lg > NEG_INF
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        s = np.exp(lg[fin] - mx, dtype=np.float32).sum(dtype=np.float32)
        lse = F32(np.log(s, dtype=np.float32) + mx)
        lp = np.where(fin, (lg - lse).astype(np.float32), NEG_INF).astype(np.float32)
        # :547-561: the timestamp block's total probability against the best text token
        ts = lp[tok.beg:]
        ts_max = ts.max() if ts.size else NEG_INF
        ts_lp = NEG_INF
        if ts_max > NEG_INF:
            tf = ts > NEG_INF
            acc = np.exp(ts[tf] - ts_max, dtype=np.float32).sum(dtype=np.float32)
            ts_lp = F32(np.log(acc, dtype=np.float32) + ts_max)
    text_max = lp[:tok.beg].max() if tok.beg > 0 else NEG_INF
    if ts_lp > text_max:
        lg[:tok.beg] = NEG_INF
    # :563-575: argmax (first index of the largest), and the largest timestamp
    best = int(np.argmax(lg)) if lg.max() > NEG_INF else 0
    tsb = lg[tok.beg:]
    tid = tok.beg + int(np.argmax(tsb)) if tsb.size and tsb.max() > NEG_INF else tok.beg
    return best, tid


@dataclass
class WindowResult:
    tokens: List[int]          # every sampled token of the window, in order
    tids: List[int]            # the most likely timestamp at each step
    result_len: int
    seek_delta: int
    has_ts: bool
    failed: bool


def new_window_state(n_audio_ctx: int) -> dict:
    return {"tokens": [], "tids": [], "seek_delta": 2 * n_audio_ctx, "has_ts": False, "result_len": 0,
            "failed": False}


def window_step(state: dict, s_id: int, s_tid: int, i: int, n_max: int, seek: int, seek_end: int,
                tok: Tokens, window: int) -> bool:
    """One token of the loop body (src/transcribe.zig:319-364) after `sample` returned
    (s_id, s_tid) at step i. Records the token and updates the window's bookkeeping in
    `state` (seek_delta, has_ts, result_len, failed). Returns True when the loop ends."""
    state["tokens"].append(s_id)
    state["tids"].append(s_tid)
    if s_id > tok.beg:
        seek_delta_new = 2 * (s_id - tok.beg)
        if state["has_ts"] and state["seek_delta"] > seek_delta_new and state["result_len"] < i:
            state["failed"] = True
            return True
        state["seek_delta"] = seek_delta_new
        state["result_len"] = i + 1
        state["has_ts"] = True
    if s_id == tok.eot or (state["has_ts"] and seek + state["seek_delta"] + 100 >= seek_end):
        if state["result_len"] == 0:
            if seek + state["seek_delta"] + 100 >= seek_end:
                state["result_len"] = i + 1
            else:
                state["failed"] = True
        return True
    if i == n_max - 1 and (state["result_len"] == 0 or state["seek_delta"] < window // 2):
        state["failed"] = True
        return True
    return False


def decode_window(forward: Callable[[List[int]], np.ndarray], prompt: List[int], seek: int, seek_end: int,
                  rules: Rules, n_text_ctx: int = 448) -> WindowResult:
    """The token loop of one window (src/transcribe.zig:292-365). `forward(tokens)` runs the
    decoder on new tokens (continuing its cache) and returns the last token's f32 logits;
    the caller has reset the decoder and set the window's audio."""
    tok = rules.tok
    n_max = n_text_ctx // 2 - 4
    window = 2 * rules.n_audio_ctx
    lg = np.array(forward(list(prompt)), np.float32)
    st = new_window_state(rules.n_audio_ctx)
    for i in range(n_max):
        is_initial = len(st["tokens"]) == 0
        s_id, s_tid = sample(lg, st["tokens"], is_initial, st["has_ts"], st["seek_delta"], rules)
        if window_step(st, s_id, s_tid, i, n_max, seek, seek_end, tok, window):
            break
        lg = np.array(forward([s_id]), np.float32)
    return WindowResult(st["tokens"], st["tids"], st["result_len"], st["seek_delta"], st["has_ts"], st["failed"])


def window_segments(res: WindowResult, seek: int, tok: Tokens, text_of: Callable[[int], str]) -> List[dict]:
    """The segments the reference emits for one window, in order: at every timestamp after
    text (src/transcribe.zig:330-339) and the trailing text (:375-382). t0/t1 in
    centiseconds after finishSpan's guard against a span running backwards (:459); the
    synthetic vocabulary has no quotes, so no span is split. A window that failed with
    nothing usable emits nothing more after its loop (:369-373)."""
    segs = []
    seg_start, seg_t0 = 0, seek
    text = ""
    n = len(res.tokens)
    for i, s_id in enumerate(res.tokens):
        if i == 0:
            seg_t0 = seek + 2 * max(res.tids[0] - tok.beg, 0)
        if s_id > tok.beg:
            if res.failed and i == n - 1 and res.result_len < i + 1:
                break  # the timestamp that went backwards ends the loop before any emit
            t1 = seek + 2 * max(res.tids[i] - tok.beg, 0)
            if text:
                segs.append(_finish(seg_t0, t1, text, res.tokens[seg_start:i + 1]))
            text = ""
            seg_t0 = t1
            seg_start = i + 1
        elif s_id < tok.eot:
            text += text_of(s_id)
    if res.failed and res.result_len == 0:
        return segs
    used = res.tokens[:res.result_len]
    if seg_start < len(used):
        text = "".join(text_of(t) for t in used[seg_start:] if t < tok.eot)
        if text:
            segs.append(_finish(seg_t0, seek + res.seek_delta, text, used[seg_start:]))
    return segs


def _finish(t0: int, t1: int, text: str, tokens: Sequence[int]) -> dict:
    if t1 < t0:
        t0 = t1
    return {"t0": t0, "t1": t1, "text": text, "tokens": list(tokens)}


def window_prompt(tok: Tokens, prompt_past: Sequence[int], prompt_tokens: Sequence[int], condition_on_previous: bool,
                  n_text_ctx: int = 448) -> List[int]:
    """The decoder prompt of a window (src/transcribe.zig:281-291): [prev, initial prompt,
    the tail of the previous windows' text] + [sot]."""
    max_prompt_ctx = n_text_ctx // 2
    prompt: List[int] = []
    past_ok = condition_on_previous and len(prompt_past) > 0
    if len(prompt_tokens) > 0 or past_ok:
        prompt.append(tok.prev)
        prompt.extend(prompt_tokens)
        if past_ok:
            budget = max_prompt_ctx - 1 - len(prompt_tokens)
            n_take = min(budget, len(prompt_past))
            prompt.extend(prompt_past[len(prompt_past) - n_take:])
    prompt.append(tok.sot)
    return prompt


def transcribe(encode_window: Callable[[int], None], forward: Callable[[List[int]], np.ndarray],
               reset: Callable[[], None], seek_end: int, rules: Rules, text_of: Callable[[int], str],
               condition_on_previous: bool = True, prompt_tokens: Sequence[int] = (),
               n_text_ctx: int = 448) -> Tuple[List[dict], List[WindowResult]]:
    """Engine.transcribe's outer loop (src/transcribe.zig:276-401) without voices, name
    learning or the prompt-echo check. `encode_window(seek)` encodes the window at mel
    frame `seek` and sets the decoder's audio; `reset()` empties the decoder's cache."""
    tok = rules.tok
    window = 2 * rules.n_audio_ctx
    prompt_past: List[int] = []
    segs: List[dict] = []
    results: List[WindowResult] = []
    seek = 0
    while seek < seek_end:
        if seek + 100 >= seek_end:
            break
        encode_window(seek)
        prompt = window_prompt(tok, prompt_past, prompt_tokens, condition_on_previous, n_text_ctx)
        prompt_fixed = 1 + len(prompt_tokens)
        reset()
        res = decode_window(forward, prompt, seek, seek_end, rules, n_text_ctx)
        results.append(res)
        segs.extend(window_segments(res, seek, tok, text_of))
        if res.failed and res.result_len == 0:
            seek += window
            prompt_past = []
            continue
        used = res.tokens[:res.result_len]
        if condition_on_previous:
            old = prompt[prompt_fixed:len(prompt) - 1] if len(prompt) > prompt_fixed else []
            prompt_past = list(old) + list(used)
        seek += res.seek_delta
    return segs, results


def synthetic_text(i: int) -> str:
    """Token text of the synthetic model files written by oracle.whisper.write_ggml (ids
    below 50257; the rest have empty text, src/model.zig:142-143)."""
    if i >= 50257:
        return ""
    return " " if i == 220 else f"<{i}>"
