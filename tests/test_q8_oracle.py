"""The Q8 restatement (oracle/q8.py) on the CPU, in the form of the reference's own test
"int8 block matches f32 within quantization error" (src/gemm.zig:365-391): a 6 x 64 input
against 7 quantized weight rows agrees with the f32 product within 0.02, and a dequantized
row agrees with its weights within 0.005. Plus the exact rounding rule of Q8.quantize
(src/gemm.zig:222-226) and the GGUF q8_0 block layout of Q8.fromQ8_0 (src/gemm.zig:233-246)."""
import numpy as np

from oracle import q8


def test_reference_form_quantization_error():
    rng = np.random.default_rng(11)
    m, n, k = 6, 7, 64
    a = (rng.random((m, k), dtype=np.float32) - 0.5).astype(np.float32)
    w = (rng.random((n, k), dtype=np.float32) - 0.5).astype(np.float16)
    q, s = q8.quantize(w)
    c = q8.linear(a, q, s)
    exact = a.astype(np.float32) @ w.astype(np.float32).T
    assert np.abs(c - exact).max() <= 0.02
    assert np.abs(q8.dequant(q, s)[2] - w[2].astype(np.float32)).max() <= 0.005


def test_rounding_is_half_away_from_zero_and_clamped():
    # one block whose absmax is 127 * 0.5: inv = 2, so v * inv lands on exact halves
    v = np.zeros((1, 32), np.float32)
    v[0, :6] = [63.5, 0.25, -0.25, 0.75, -0.75, 1.25]
    q, s = q8.quantize(v)
    assert s[0, 0] == np.float32(63.5) / np.float32(127.0)
    assert list(q[0, :6]) == [127, 1, -1, 2, -2, 3]  # 0.5 -> 1, -0.5 -> -1, 1.5 -> 2, 2.5 -> 3
    z, sz = q8.quantize(np.zeros((2, 64), np.float32))
    assert not z.any() and not sz.any()


def test_from_q8_0_layout():
    rng = np.random.default_rng(3)
    n, k = 3, 64
    qs = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    sc = rng.random((n, k // 32), dtype=np.float32).astype(np.float16)
    blob = b"".join(sc[i, b].tobytes() + qs[i, b * 32:(b + 1) * 32].tobytes() for i in range(n) for b in range(k // 32))
    q, s = q8.from_q8_0(blob, n, k)
    assert np.array_equal(q, qs) and np.array_equal(s, sc.astype(np.float32))


def test_linear_with_bias_matches_dequantized_product():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 96), dtype=np.float32)
    q, s = q8.quantize(rng.standard_normal((10, 96), dtype=np.float32))
    b = rng.standard_normal(10, dtype=np.float32)
    want = x.astype(np.float64) @ q8.dequant(q, s).astype(np.float64).T + b
    np.testing.assert_allclose(q8.linear(x, q, s, b), want, rtol=1e-6, atol=1e-6)
