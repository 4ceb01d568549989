"""Qwen2 pieces around the attention call (src/llm.zig:168-238), restated in numpy.

TEST INFRASTRUCTURE ONLY.

- `rope_tables`: cos/sin [n_ctx][d/2]; inverse frequencies base^(-2i/d) and the angle
  computed in float64, then cast to float32 (src/llm.zig:128-137).
- `rope`: NeoX rotation, pairs (k, k + d/2), in float32 with separately rounded products
  and differences (src/llm.zig:221-238).
- `rope_and_append`: rotate q and k at positions n_past.., scatter k into the transposed
  cache [n_head_kv][d][n_ctx] and copy v rows into [n_ctx][n_head_kv*d]
  (src/llm.zig:182-190).
- `attention_call`: the shape the model passes to attentionEx (src/llm.zig:191-202).
"""
from __future__ import annotations

import numpy as np

from . import attention as A


def rope_tables(n_ctx: int, d: int, base: float):
    half = d // 2
    cos = np.empty((n_ctx, half), np.float32)
    sin = np.empty((n_ctx, half), np.float32)
    for i in range(half):
        inv = 1.0 / np.power(np.float64(base), np.float64(2 * i) / np.float64(d))
        ang = np.arange(n_ctx, dtype=np.float64) * inv
        cos[:, i] = np.cos(ang).astype(np.float32)
        sin[:, i] = np.sin(ang).astype(np.float32)
    return cos, sin


def rope(x: np.ndarray, n: int, heads: int, d: int, n_past: int, cos, sin) -> np.ndarray:
    """In-place NeoX RoPE on x[n][heads*d] (float32)."""
    half = d // 2
    x = x.reshape(n, heads, d)
    c = cos[n_past:n_past + n][:, None, :]
    s = sin[n_past:n_past + n][:, None, :]
    a = x[:, :, :half].copy()
    b = x[:, :, half:].copy()
    x[:, :, :half] = (a * c).astype(np.float32) - (b * s).astype(np.float32)
    x[:, :, half:] = (a * s).astype(np.float32) + (b * c).astype(np.float32)
    return x.reshape(n, heads * d)


def rope_and_append(q, k, v, cache_kt, cache_v, cos, sin, n_past, n_head, n_head_kv, d):
    n = q.size // (n_head * d)
    q = np.array(q, np.float32).reshape(n, n_head * d)
    k = np.array(k, np.float32).reshape(n, n_head_kv * d)
    v = np.asarray(v, np.float32).reshape(n, n_head_kv * d)
    rope(q, n, n_head, d, n_past, cos, sin)
    rope(k, n, n_head_kv, d, n_past, cos, sin)
    n_ctx = cache_kt.size // (n_head_kv * d)
    kt = cache_kt.reshape(n_head_kv, d, n_ctx)
    for i in range(n):
        for h in range(n_head_kv):
            kt[h, :, n_past + i] = k[i, h * d:(h + 1) * d]
    cache_v.reshape(n_ctx, n_head_kv * d)[n_past:n_past + n] = v
    return q, cache_kt, cache_v


def attention_call(n: int, n_kv: int, n_head: int, n_head_kv: int, d: int, n_ctx: int) -> A.AttnShape:
    ne = n_head * d
    return A.AttnShape(n, n_kv, n_head, n_head_kv, d, ne, n_head_kv * d, ne, True, n_ctx)
