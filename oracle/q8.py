"""Q8 weights and the linear layer over them (src/gemm.zig:188-351, src/ops.zig:243-306),
restated in numpy.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA Q8 kernels, never the product path.

- `quantize`: Q8.quantize (src/gemm.zig:208-230): rows of k split into blocks of 32, each
  with scale = absmax / 127 (f32) and q = clamp(round(v * (127 / absmax)), -127, 127), the
  product v * inv rounded to f32 and then rounded half away from zero (Zig's @round).
- `dequant`: Q8.row (src/gemm.zig:254-263): q * scale per block.
- `from_q8_0`: Q8.fromQ8_0 (src/gemm.zig:233-246): GGUF q8_0 blocks (an f16 scale then 32
  int8) to the same int8 rows and f32 scales.
- `linear`: ops.linear with Q8 weights (src/ops.zig:280-306 -> gemm.ntBlockQ,
  src/gemm.zig:268-351): out[m][n] = sum over blocks b of scale[n][b] * (x[m] . q[n]
  over block b), plus bias[n]. Accumulated in float64 here; the reference accumulates in f32
  vectors, so results agree to f32 rounding, not bit for bit.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

BLOCK = 32


def _round_half_away(r: np.ndarray) -> np.ndarray:
    """Round to the nearest integer, ties away from zero, exactly (no 0.5 added)."""
    t = np.trunc(r)
    frac = np.abs(r - t)  # exact for f32 inputs
    return t + np.sign(r) * (frac >= np.float32(0.5))


def quantize(w: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    w = np.asarray(w).astype(np.float32)
    n, k = w.shape
    assert k % BLOCK == 0
    blk = w.reshape(n, k // BLOCK, BLOCK)
    amax = np.abs(blk).max(-1)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    inv = np.where(amax > 0, np.float32(127.0) / np.where(amax > 0, amax, np.float32(1)), np.float32(0))
    inv = inv.astype(np.float32)
    r = (blk * inv[..., None]).astype(np.float32)
    q = np.clip(_round_half_away(r), -127, 127).astype(np.int8)
    return q.reshape(n, k), scale


def dequant(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    n, k = q.shape
    return (q.reshape(n, k // BLOCK, BLOCK).astype(np.float32) * scale[..., None]).reshape(n, k).astype(np.float32)


def from_q8_0(data: bytes, n: int, k: int) -> Tuple[np.ndarray, np.ndarray]:
    nb = k // BLOCK
    raw = np.frombuffer(data, dtype=np.uint8, count=n * nb * 34).reshape(n * nb, 34)
    scale = raw[:, :2].copy().view(np.float16).astype(np.float32).reshape(n, nb)
    q = raw[:, 2:].copy().view(np.int8).reshape(n, k)
    return q, scale


def linear(x: np.ndarray, q: np.ndarray, scale: np.ndarray, bias: Optional[np.ndarray] = None) -> np.ndarray:
    """out = x . W^T (+ bias) with W = q * scale per block of 32, summed in float64 (the
    reference's per-block f32 dots scaled by the block's scale, src/gemm.zig:268-351, to
    well below f32 rounding). Row chunks of W go through one float64 matrix product each."""
    x = np.asarray(x, np.float32)
    m, k = x.shape
    n = q.shape[0]
    if m <= 8:
        # a few rows: per-block dots, then the scales (no float64 copy of the weights)
        xb = x.reshape(m, k // BLOCK, BLOCK).astype(np.float64)
        qb = q.reshape(n, k // BLOCK, BLOCK).astype(np.float64)
        t = np.einsum("mbi,nbi->mnb", xb, qb)
        out = (t * scale.astype(np.float64)[None]).sum(-1)
        if bias is not None:
            out = out + np.asarray(bias, np.float64)[None]
        return out.astype(np.float32)
    x64 = x.astype(np.float64)
    out = np.empty((m, n), np.float64)
    step = max(1, (1 << 24) // max(k, 1))  # ~128 MB of float64 weights per chunk
    for n0 in range(0, n, step):
        n1 = min(n, n0 + step)
        w = (q[n0:n1].reshape(n1 - n0, k // BLOCK, BLOCK).astype(np.float64)
             * scale[n0:n1].astype(np.float64)[..., None]).reshape(n1 - n0, k)
        out[:, n0:n1] = x64 @ w.T
    if bias is not None:
        out = out + np.asarray(bias, np.float64)[None]
    return out.astype(np.float32)
