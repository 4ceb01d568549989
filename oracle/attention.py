"""Numpy restatement of the reference attention (src/ops.zig:464-605).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never the product path.

The order of operations follows the reference:
  1. K is transposed per kv head into KT[hk][d][n_kv_pad], zero padded
     (AttnJob.transpose, ops.zig:505-515), unless the caller keeps keys transposed
     (`kt_stride`, ops.zig:488-491).
  2. Tasks are (head, block of q_block=64 query rows) (ops.zig:517-541, 584-589).
  3. S = Q_h . KT over `cols` = n_kv rounded up to the vector width (gemm.pvBlock,
     gemm.zig:139-186), scaled by 1/sqrt(d) after the dot (ops.zig:533-535).
  4. Row softmax over `limit` columns: causal limit n_kv - n_q + row + 1
     (ops.zig:534), max subtracted, divided by the sum (softmaxRow, ops.zig:442-462);
     columns past the limit are zeroed.
  5. O = S . V_h over all n_kv rows (ops.zig:539-540).
Head h reads kv head h // (n_head // n_head_kv) (ops.zig:521).

Everything is float32 like the reference; summation order inside the dot products is
numpy's, which differs from the reference's FMA chains by rounding only (~1e-7 relative).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

# Reference vector width on AVX-512 hosts (gemm.zig:15-23). It only changes the zero
# padding of KT and the number of score columns computed; results do not depend on it.
V = 16
Q_BLOCK = 64  # ops.zig:473


@dataclass
class AttnShape:
    """Mirror of `AttnShape` (ops.zig:477-492). Strides are in floats."""

    n_q: int
    n_kv: int
    n_head: int
    n_head_kv: int
    d: int
    q_stride: int
    kv_stride: int
    out_stride: int
    causal: bool
    kt_stride: Optional[int] = None

    def check(self) -> None:
        assert self.n_head_kv > 0 and self.n_head % self.n_head_kv == 0
        assert self.d > 0
        if self.causal:
            assert self.n_kv >= self.n_q
        if self.kt_stride is not None:
            assert self.kt_stride >= self.n_kv


def mha_shape(n_q: int, n_kv: int, n_state: int, n_head: int, causal: bool) -> AttnShape:
    """The shape `ops.attention` builds (ops.zig:593-605)."""
    return AttnShape(n_q, n_kv, n_head, n_head, n_state // n_head, n_state, n_state, n_state, causal)


def softmax_row(x: np.ndarray) -> np.ndarray:
    """softmaxRow (ops.zig:442-462): max-subtract, exp, divide by the sum (f32)."""
    x = x.astype(np.float32, copy=False)
    if x.size == 0:
        return x
    mx = np.max(x)
    e = np.exp(np.maximum(x - mx, np.float32(-87.3)), dtype=np.float32)
    s = np.float32(e.sum(dtype=np.float32))
    return e * (np.float32(1.0) / s)


def attention_ex(q: np.ndarray, k: np.ndarray, v: np.ndarray, sh: AttnShape,
                 out: Optional[np.ndarray] = None) -> np.ndarray:
    """attentionEx (ops.zig:562-590). q, k, v, out are flat float32 arrays.

    Layouts: q[n_q][q_stride] (head h at columns h*d..), v[n_kv][kv_stride] (kv head hk
    at hk*d..), out[n_q][out_stride]; k is [n_kv][kv_stride] or, with kt_stride,
    [n_head_kv][d][kt_stride].
    """
    sh.check()
    d = sh.d
    q = np.asarray(q, dtype=np.float32).reshape(-1)
    k = np.asarray(k, dtype=np.float32).reshape(-1)
    v = np.asarray(v, dtype=np.float32).reshape(-1)
    if out is None:
        out = np.zeros(max(sh.n_q, 1) * sh.out_stride, dtype=np.float32)
    if sh.n_q == 0:
        return out
    group = sh.n_head // sh.n_head_kv
    cols = (sh.n_kv + V - 1) // V * V
    # KT[hk][p][t]
    if sh.kt_stride is None:
        n_kv_pad = cols
        kt = np.zeros((sh.n_head_kv, d, n_kv_pad), dtype=np.float32)
        if sh.n_kv:
            kr = k[: (sh.n_kv - 1) * sh.kv_stride + sh.n_head_kv * d]
            for hk in range(sh.n_head_kv):
                rows = np.stack([kr[t * sh.kv_stride + hk * d: t * sh.kv_stride + (hk + 1) * d]
                                 for t in range(sh.n_kv)])
                kt[hk, :, : sh.n_kv] = rows.T
    else:
        n_kv_pad = sh.kt_stride
        kt = k[: sh.n_head_kv * d * n_kv_pad].reshape(sh.n_head_kv, d, n_kv_pad)
        cols = min(cols, n_kv_pad)
    vrows = None
    if sh.n_kv:
        vrows = np.stack([v[t * sh.kv_stride: t * sh.kv_stride + sh.n_head_kv * d]
                          for t in range(sh.n_kv)])  # [n_kv][Hkv*d]
    qrows = np.stack([q[i * sh.q_stride: i * sh.q_stride + sh.n_head * d] for i in range(sh.n_q)])
    scl = np.float32(1.0) / np.sqrt(np.float32(d), dtype=np.float32)
    o_all = np.zeros((sh.n_q, sh.n_head * d), dtype=np.float32)
    for h in range(sh.n_head):
        hk = h // group
        for q0 in range(0, sh.n_q, Q_BLOCK):
            q1 = min(q0 + Q_BLOCK, sh.n_q)
            qh = qrows[q0:q1, h * d:(h + 1) * d]
            s = qh @ kt[hk, :, :cols]  # [m][cols]
            for i in range(q1 - q0):
                limit = sh.n_kv - sh.n_q + q0 + i + 1 if sh.causal else sh.n_kv
                row = s[i, :limit] * scl
                s[i, :limit] = softmax_row(row)
                s[i, limit:] = 0
            if sh.n_kv:
                o_all[q0:q1, h * d:(h + 1) * d] = s[:, : sh.n_kv] @ vrows[:, hk * d:(hk + 1) * d]
    for i in range(sh.n_q):
        out[i * sh.out_stride: i * sh.out_stride + sh.n_head * d] = o_all[i]
    return out


def attention(q, k, v, n_q, n_kv, n_state, n_head, causal, out=None):
    """ops.attention (ops.zig:593-605)."""
    return attention_ex(q, k, v, mha_shape(n_q, n_kv, n_state, n_head, causal), out)


def naive_attention(q, k, v, n_q, n_kv, n_state, n_head, causal):
    """The naive loop of the reference's own unit test (ops.zig:655-704), vectorised per
    row: scores divided by sqrt(d), exp(s - max), probabilities s / sum times V."""
    d = n_state // n_head
    q = np.asarray(q, np.float32).reshape(n_q, n_state)
    k = np.asarray(k, np.float32).reshape(n_kv, n_state)
    v = np.asarray(v, np.float32).reshape(n_kv, n_state)
    out = np.zeros((n_q, n_state), np.float32)
    for h in range(n_head):
        sl = slice(h * d, (h + 1) * d)
        for i in range(n_q):
            limit = n_kv - n_q + i + 1 if causal else n_kv
            sc = (k[:limit, sl] @ q[i, sl]) / np.sqrt(np.float32(d))
            e = np.exp(sc - sc.max())
            out[i, sl] = (e / e.sum()) @ v[:limit, sl]
    return out.reshape(-1)


def attention_batched(q, k, v, causal: bool, n_kv_valid=None):
    """Batched float64 reference for large parity cases (any layout converted to
    [B][H][n][d]); used where the per-row loop above would take too long. GQA is
    expressed by k/v having fewer heads. Returns float64 [B][H][n_q][d]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, H, n_q, d = q.shape
    Hk = k.shape[1]
    g = H // Hk
    n_kv = k.shape[2]
    out = np.empty_like(q)
    for hk in range(Hk):
        qs = q[:, hk * g:(hk + 1) * g]  # [B][g][n_q][d]
        s = np.einsum("bgid,bjd->bgij", qs, k[:, hk]) / np.sqrt(d)
        if causal:
            i = np.arange(n_q)[:, None]
            j = np.arange(n_kv)[None, :]
            s = np.where(j <= n_kv - n_q + i, s, -np.inf)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[:, hk * g:(hk + 1) * g] = np.einsum("bgij,bjd->bgid", p, v[:, hk])
    return out
