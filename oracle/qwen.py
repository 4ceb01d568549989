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
- `rms_norm`, `silu_mul`: ops.rmsNorm (src/ops.zig:408-425) and ops.siluMul
  (src/ops.zig:435-440) in float32; the sum of squares is accumulated in float64 here
  (the reference sums f32 vectors), so results agree to f32 rounding.
- `embed`: Q8.row (src/gemm.zig:256-263) of each token, bit for bit.
- `layer_forward`, `forward`: Model.forward (src/llm.zig:169-216) on numpy weights, the
  caches of one sequence per batch item.
- `greedy`: Model.penalize then Model.argmax (src/llm.zig:268-273, 313-321).
- `make_model`: a seeded random Qwen2 model in Q8 (weights N(0, 0.02^2), quantized with
  Q8.quantize; norm gains near 1) for the tests.
"""
from __future__ import annotations

import numpy as np

from . import attention as A
from . import q8


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


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """x / sqrt(mean(x^2) + eps) * w over the last axis (src/ops.zig:408-425), float32."""
    x = np.asarray(x, np.float32)
    n = x.shape[-1]
    ss = (x.astype(np.float64) ** 2).sum(-1).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(ss / np.float32(n) + np.float32(eps))).astype(np.float32)
    return ((x * inv[..., None]).astype(np.float32) * np.asarray(w, np.float32)).astype(np.float32)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """gate / (1 + exp(-gate)) * up (src/ops.zig:435-440), float32."""
    g = np.asarray(g, np.float32)
    return ((g / (np.float32(1.0) + np.exp(-g))).astype(np.float32) * np.asarray(u, np.float32)).astype(np.float32)


def embed(q: np.ndarray, scales: np.ndarray, tokens) -> np.ndarray:
    """Q8.row (src/gemm.zig:256-263) for each token: q * scale in float32."""
    t = np.asarray(tokens).reshape(-1)
    return q8.dequant(q[t], scales[t])


def layer_forward(x: np.ndarray, L: dict, kt: np.ndarray, v: np.ndarray, n_past: int, n_head: int,
                  n_head_kv: int, d: int, eps: float, cos, sin) -> None:
    """One layer of Model.forward (src/llm.zig:177-210) for one sequence, in place on x
    [n][n_embd] and on this layer's caches kt [n_head_kv*d*n_ctx], v [n_ctx*n_head_kv*d]."""
    n, ne = x.shape
    n_ctx = kt.size // (n_head_kv * d)
    h = rms_norm(x, L["attn_norm"], eps)
    q = q8.linear(h, *L["wq"], L.get("bq"))
    k = q8.linear(h, *L["wk"], L.get("bk"))
    vv = q8.linear(h, *L["wv"], L.get("bv"))
    qr, _, _ = rope_and_append(q, k, vv, kt, v, cos, sin, n_past, n_head, n_head_kv, d)
    sh = attention_call(n, n_past + n, n_head, n_head_kv, d, n_ctx)
    attn = A.attention_ex(qr.reshape(-1), kt, v, sh).reshape(n, ne)
    x += q8.linear(attn, *L["wo"])
    h = rms_norm(x, L["ffn_norm"], eps)
    g = silu_mul(q8.linear(h, *L["w_gate"]), q8.linear(h, *L["w_up"]))
    x += q8.linear(g, *L["w_down"])


def forward(model: dict, tokens: np.ndarray, caches, n_past: int):
    """Model.forward (src/llm.zig:169-216) for every sequence: tokens [B][n]; caches[b][l] =
    (kt, v) numpy arrays updated in place. Returns (x [B][n][n_embd], logits [B][n_vocab] of
    each sequence's last token)."""
    tokens = np.asarray(tokens)
    B, n = tokens.shape
    cfg = model["cfg"]
    xs, logits = [], []
    for b in range(B):
        x = embed(*model["embd"], tokens[b])
        for li, L in enumerate(model["layers"]):
            kt, v = caches[b][li]
            layer_forward(x, L, kt, v, n_past, cfg["n_head"], cfg["n_head_kv"], cfg["d"], cfg["eps"],
                          model["cos"], model["sin"])
        h = rms_norm(x[n - 1:n], model["output_norm"], cfg["eps"])
        logits.append(q8.linear(h, *model["output"])[0])
        xs.append(x)
    return np.stack(xs), np.stack(logits)


def greedy(logits: np.ndarray, recent, window: int = 64, penalty: float = 1.1) -> int:
    """Model.penalize then Model.argmax (src/llm.zig:268-273, 313-321) on one row of logits,
    penalized in place: repeats are penalized again; the first index of the largest value
    wins; NaN never wins, and a NaN in column 0 gives 0."""
    row = logits
    if penalty > 1.0:
        recent = list(recent)
        for t in recent[max(0, len(recent) - window):]:
            val = row[t]
            row[t] = np.float32(val / np.float32(penalty)) if val > 0 else np.float32(val * np.float32(penalty))
    if np.isnan(row[0]):
        return 0
    return int(np.argmax(np.where(np.isnan(row), -np.inf, row)))


def make_model(seed: int, n_layer: int, n_vocab: int, n_head: int, n_head_kv: int, d: int, n_ff: int, n_ctx: int,
               rope_base: float = 1e6, eps: float = 1e-6, bias: bool = True, tied: bool = True) -> dict:
    """A random Qwen2 model in the reference's formats: Q8 matrices as (q, scales), f32
    norms and biases, RoPE tables."""
    rng = np.random.default_rng(seed)
    ne = n_head * d
    kvw = n_head_kv * d

    def mat(n, k):
        return q8.quantize((rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32))

    def vec(n, mean, sd):
        return (mean + rng.standard_normal(n, dtype=np.float32) * np.float32(sd)).astype(np.float32)

    layers = []
    for _ in range(n_layer):
        layers.append({
            "attn_norm": vec(ne, 1.0, 0.1), "wq": mat(ne, ne), "wk": mat(kvw, ne), "wv": mat(kvw, ne),
            "bq": vec(ne, 0.0, 0.1) if bias else None, "bk": vec(kvw, 0.0, 0.1) if bias else None,
            "bv": vec(kvw, 0.0, 0.1) if bias else None, "wo": mat(ne, ne), "ffn_norm": vec(ne, 1.0, 0.1),
            "w_gate": mat(n_ff, ne), "w_up": mat(n_ff, ne), "w_down": mat(ne, n_ff),
        })
    embd = mat(n_vocab, ne)
    cos, sin = rope_tables(n_ctx, d, rope_base)
    return {
        "cfg": dict(n_layer=n_layer, n_vocab=n_vocab, n_head=n_head, n_head_kv=n_head_kv, d=d, n_ff=n_ff,
                    n_ctx=n_ctx, eps=eps, rope_base=rope_base),
        "layers": layers, "embd": embd, "output": embd if tied else mat(n_vocab, ne),
        "output_norm": vec(ne, 1.0, 0.1), "cos": cos, "sin": sin,
    }


def new_caches(model: dict, n_batch: int):
    """Zeroed (kt, v) caches per sequence and layer, as the reference allocates them
    (src/llm.zig:124-127)."""
    c = model["cfg"]
    size = c["n_head_kv"] * c["d"] * c["n_ctx"]
    return [[(np.zeros(size, np.float32), np.zeros(size, np.float32)) for _ in range(c["n_layer"])]
            for _ in range(n_batch)]
