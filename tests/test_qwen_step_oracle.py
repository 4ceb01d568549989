"""The oracle's Qwen2 decode-step pieces (oracle/qwen.py; src/llm.zig:169-216, 268-321,
src/ops.zig:408-440) on the CPU: the formulas against float64 restatements, the penalty and
argmax rules against hand-worked rows, and Model.forward's cache handling through the
chunking invariance the reference relies on when it feeds a prompt in batches
(src/llm.zig:257-266)."""
import numpy as np

from oracle import q8, qwen


def test_rms_norm_formula():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 96), dtype=np.float32)
    w = rng.standard_normal(96, dtype=np.float32)
    got = qwen.rms_norm(x, w, 1e-6)
    x64 = x.astype(np.float64)
    want = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-7)
    assert got.dtype == np.float32


def test_silu_mul_formula():
    rng = np.random.default_rng(1)
    g = rng.standard_normal(1000, dtype=np.float32) * 4
    u = rng.standard_normal(1000, dtype=np.float32)
    want = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u
    np.testing.assert_allclose(qwen.silu_mul(g, u), want, rtol=2e-6, atol=1e-7)


def test_embed_is_q8_row():
    rng = np.random.default_rng(2)
    q, s = q8.quantize(rng.standard_normal((50, 64), dtype=np.float32))
    rows = qwen.embed(q, s, [3, 0, 49, 3])
    full = q8.dequant(q, s)
    assert np.array_equal(rows, full[[3, 0, 49, 3]])


def test_greedy_penalty_and_ties():
    row = np.array([0.5, 2.0, -1.0, 2.0, 1.9], np.float32)
    # ties: the first index of the maximum
    assert qwen.greedy(row.copy(), [], penalty=1.0) == 1
    # token 1 penalized once: 2.0 / 1.1 < 2.0 at index 3
    assert qwen.greedy(row.copy(), [1], penalty=1.1) == 3
    # repeats are penalized again: 1 and 3 twice each, 4 wins
    r = row.copy()
    assert qwen.greedy(r, [1, 3, 1, 3], penalty=1.1) == 4
    assert r[1] == np.float32(np.float32(2.0 / np.float32(1.1)) / np.float32(1.1))
    # negative logits are multiplied
    r = row.copy()
    qwen.greedy(r, [2], penalty=1.5)
    assert r[2] == np.float32(-1.5)
    # the window keeps only the last entries
    assert qwen.greedy(row.copy(), [1, 3, 1], window=1, penalty=1.1) == 3


def test_greedy_nan_rules():
    assert qwen.greedy(np.array([np.nan, 1.0, 2.0], np.float32), []) == 0
    assert qwen.greedy(np.array([0.0, np.nan, -2.0], np.float32), []) == 0
    assert qwen.greedy(np.array([-1.0, np.nan, 3.0], np.float32), []) == 2
    assert qwen.greedy(np.array([-np.inf, -np.inf], np.float32), []) == 0


def test_forward_chunking_invariance():
    """Feeding a prompt whole or in chunks gives the same hidden states and logits: the
    caches and positions carry the state between calls."""
    m = qwen.make_model(3, n_layer=2, n_vocab=300, n_head=4, n_head_kv=2, d=32, n_ff=256, n_ctx=32)
    toks = np.random.default_rng(4).integers(0, 300, (2, 11))
    c1 = qwen.new_caches(m, 2)
    qwen.forward(m, toks[:, :5], c1, 0)
    x_b, l_b = qwen.forward(m, toks[:, 5:], c1, 5)
    c2 = qwen.new_caches(m, 2)
    x_a, l_a = qwen.forward(m, toks, c2, 0)
    np.testing.assert_allclose(x_b, x_a[:, 5:], atol=1e-6)
    np.testing.assert_allclose(l_b, l_a, atol=1e-6)
    for b in range(2):
        for li in range(2):
            np.testing.assert_array_equal(c1[b][li][0], c2[b][li][0])
