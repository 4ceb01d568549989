"""CPU checks of the oracle itself (no GPU): the numpy restatement of the reference
attention and the C restatement against the naive loop of the reference's own unit test
(src/ops.zig:655-704), against each other, and on the reference's edge cases."""
import numpy as np
import pytest

from oracle import attention as A
from oracle import cref, qwen


def rnd(rng, n):
    return (rng.random(n, dtype=np.float32) - 0.5).astype(np.float32)


@pytest.mark.parametrize("causal", [False, True])
def test_reference_unit_test_restated(causal):
    """src/ops.zig:655-704: n_q=70, n_kv=90, 2 heads, d = 2V (V=16), abs tol 1e-4."""
    rng = np.random.default_rng(9)
    n_q, n_kv, H = 70, 90, 2
    ns = 2 * A.V * H
    q, k, v = rnd(rng, n_q * ns), rnd(rng, n_kv * ns), rnd(rng, n_kv * ns)
    naive = A.naive_attention(q, k, v, n_q, n_kv, ns, H, causal)
    np.testing.assert_allclose(A.attention(q, k, v, n_q, n_kv, ns, H, causal), naive, atol=1e-4, rtol=0)
    np.testing.assert_allclose(cref.attention_ex(q, k, v, A.mha_shape(n_q, n_kv, ns, H, causal)), naive,
                               atol=1e-4, rtol=0)


@pytest.mark.parametrize("n_q,n_kv,H,Hkv,d,causal,kt", [
    (1, 1, 1, 1, 16, False, None),
    (1, 17, 2, 2, 32, True, None),
    (3, 65, 4, 2, 64, True, None),
    (65, 129, 2, 1, 64, False, None),
    (9, 300, 14, 2, 64, True, 320),
    (2, 100, 12, 2, 128, True, 112),
])
def test_numpy_vs_c_restatement(n_q, n_kv, H, Hkv, d, causal, kt):
    rng = np.random.default_rng(n_q + n_kv + d)
    sh = A.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, causal, kt)
    q = rnd(rng, n_q * H * d)
    k = rnd(rng, Hkv * d * kt) if kt else rnd(rng, n_kv * Hkv * d)
    v = rnd(rng, n_kv * Hkv * d)
    a = A.attention_ex(q, k, v, sh)
    b = cref.attention_ex(q, k, v, sh)
    np.testing.assert_allclose(a, b, atol=1e-5, rtol=0)


def test_batched_float64_reference_agrees():
    rng = np.random.default_rng(4)
    B, H, Hkv, n_q, n_kv, d = 2, 6, 2, 5, 40, 32
    q = rng.standard_normal((B, H, n_q, d))
    k = rng.standard_normal((B, Hkv, n_kv, d))
    v = rng.standard_normal((B, Hkv, n_kv, d))
    got = A.attention_batched(q, k, v, causal=True)
    for b in range(B):
        qf = q[b].transpose(1, 0, 2).reshape(-1).astype(np.float32)
        kf = k[b].transpose(1, 0, 2).reshape(-1).astype(np.float32)
        vf = v[b].transpose(1, 0, 2).reshape(-1).astype(np.float32)
        sh = A.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True)
        want = A.attention_ex(qf, kf, vf, sh).reshape(n_q, H, d).transpose(1, 0, 2)
        np.testing.assert_allclose(got[b], want, atol=1e-5)


def test_empty_rows_are_zero():
    """n_kv = 0: the reference's softmax of an empty row and P.V over zero rows give 0."""
    sh = A.mha_shape(2, 0, 64, 2, False)
    out = A.attention_ex(np.ones(128, np.float32), np.zeros(0, np.float32), np.zeros(0, np.float32), sh)
    assert np.all(out == 0)


def test_causal_requires_enough_keys():
    with pytest.raises(AssertionError):
        A.attention_ex(np.zeros(64 * 3), np.zeros(64 * 2), np.zeros(64 * 2), A.mha_shape(3, 2, 64, 1, True))


def test_rope_tables_are_f64_then_f32():
    cos, sin = qwen.rope_tables(8, 64, 1e6)
    ang = 7 * (1.0 / 1e6 ** (2 * 5 / 64))
    assert cos[7, 5] == np.float32(np.cos(ang)) and sin[7, 5] == np.float32(np.sin(ang))


def test_rope_and_append_layout():
    """Scatter into the transposed cache: cache_kt[h][p][n_past+i] = k_rot[i][h*d+p]."""
    rng = np.random.default_rng(1)
    n, n_past, H, Hkv, d, n_ctx = 3, 4, 4, 2, 8, 16
    cos, sin = qwen.rope_tables(n_ctx, d, 1e6)
    q = rng.standard_normal(n * H * d).astype(np.float32)
    k = rng.standard_normal(n * Hkv * d).astype(np.float32)
    v = rng.standard_normal(n * Hkv * d).astype(np.float32)
    kt = np.zeros(Hkv * d * n_ctx, np.float32)
    vc = np.zeros(n_ctx * Hkv * d, np.float32)
    qr, kt, vc = qwen.rope_and_append(q, k, v, kt, vc, cos, sin, n_past, H, Hkv, d)
    kr = qwen.rope(k.copy().reshape(n, Hkv * d), n, Hkv, d, n_past, cos, sin)
    kt3 = kt.reshape(Hkv, d, n_ctx)
    for i in range(n):
        for h in range(Hkv):
            assert np.array_equal(kt3[h, :, n_past + i], kr[i, h * d:(h + 1) * d])
    assert np.array_equal(vc.reshape(n_ctx, -1)[n_past:n_past + n], v.reshape(n, -1))
    # position 0 is the identity rotation
    assert np.array_equal(qwen.rope(q.copy().reshape(n, -1), n, H, d, 0, cos, sin)[0], q.reshape(n, -1)[0])
