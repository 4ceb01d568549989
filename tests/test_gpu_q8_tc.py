"""The tcgen05 Q8 product (csrc/q8_tc.cu) against the oracle (oracle/q8.py; gemm.ntBlockQ,
src/gemm.zig:268-351) and against the register-tiled CUDA-core kernel it replaces for 16 or
more rows with k a multiple of 64.

Each 32-wide block dot is formed on the tensor cores from exact operands (int8 weights in
bf16, each f32 activation split into three bf16 pieces that sum to it exactly), so the only
roundings are f32 sums: the products are held to the same bound as the other Q8 kernels,
2e-6 of the sum of |terms| of each output (about 16 f32 ulps). Covered: every epilogue
(store + bias, add into out, tanh GELU, the SiLU pair, the Qwen2 q/k/v + RoPE pair here; the
Whisper decoder's q/k/v product in tests/test_gpu_dec_step.py at 16 windows), the 64-row
and 128-row tile forms, partial row and column tiles, k
split over clusters of CTAs (deterministic), activations over a wide dynamic range, and the
process-wide switch between the two kernels (which give different roundings, so the
tensor-core kernel is seen to run). The module runs with the switch at "always" (every covered
shape on the tcgen05 kernel); the default's routing by size is checked on its own."""
import numpy as np
import pytest

from oracle import q8
from oracle import qwen
from oracle import whisper as W
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    prev = ops.q8_tensor_cores("always")
    yield torch, ops
    ops.q8_tensor_cores(prev)


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def rand_q8(rng, n, k):
    return q8.quantize((rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32))


def bound(x, qs):
    return np.abs(x).astype(np.float64) @ np.abs(q8.dequant(*qs)).astype(np.float64).T


def check(got, want, mag):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert (err <= 2e-6 * mag + 1e-30).all(), float((err / (mag + 1e-30)).max())


SHAPES = [(16, 1, 64), (17, 100, 128), (64, 128, 896), (65, 129, 1536), (200, 896, 896), (64, 4864, 896),
          (32, 1536, 8960), (1500, 512, 512), (48, 8192, 512)]


@pytest.mark.parametrize("tc", [True, False], ids=["tcgen05", "cuda_cores"])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_store_bias_matches_oracle(env, m, n, k, tc):
    torch, ops = env
    rng = np.random.default_rng(m * 7 + n + k)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rand_q8(rng, n, k)
    b = rng.standard_normal(n, dtype=np.float32)
    ops.q8_tensor_cores("always" if tc else False)
    try:
        got = ops.linear_q8(dev(torch, x), dev(torch, w[0]), dev(torch, w[1]), dev(torch, b)).cpu().numpy()
    finally:
        ops.q8_tensor_cores("always")
    check(got, q8.linear(x, *w, b), bound(x, w) + np.abs(b))


@pytest.mark.parametrize("m,n,k", [(16, 896, 896), (64, 1536, 8960), (200, 100, 256)])
def test_add_into_out(env, m, n, k):
    torch, ops = env
    rng = np.random.default_rng(m + 3 * n + k)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rand_q8(rng, n, k)
    r = rng.standard_normal((m, n), dtype=np.float32)
    out = dev(torch, r)
    ops.linear_q8_add(dev(torch, x), dev(torch, w[0]), dev(torch, w[1]), out)
    check(out.cpu().numpy(), r + q8.linear(x, *w), bound(x, w) + np.abs(r))


@pytest.mark.parametrize("m,n,k", [(16, 2048, 512), (100, 1536, 384), (1500, 1536, 384)])
def test_gelu(env, m, n, k):
    torch, ops = env
    rng = np.random.default_rng(m + n + 5 * k)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rand_q8(rng, n, k)
    b = rng.standard_normal(n, dtype=np.float32)
    got = ops.linear_q8_gelu(dev(torch, x), dev(torch, w[0]), dev(torch, w[1]), dev(torch, b)).cpu().numpy()
    pre = q8.linear(x, *w, b)
    want = W.gelu(pre)
    # the product's error through gelu' (at most 1.13) plus tanh's own few ulps
    tol = 2e-6 * 1.13 * (bound(x, w) + np.abs(b)) + 2e-6 * np.abs(want) + 1e-6
    assert (np.abs(got - want) <= tol).all()


@pytest.mark.parametrize("m,n,k", [(16, 101, 256), (64, 4864, 896), (200, 1000, 1536), (33, 8960, 1536)])
def test_silu_pair(env, m, n, k):
    torch, ops = env
    rng = np.random.default_rng(m * 11 + n + k)
    x = rng.standard_normal((m, k), dtype=np.float32)
    g, u = rand_q8(rng, n, k), rand_q8(rng, n, k)
    got = ops.linear_q8_silu_mul(dev(torch, x), (dev(torch, g[0]), dev(torch, g[1])),
                                 (dev(torch, u[0]), dev(torch, u[1]))).cpu().numpy()
    gv, uv = q8.linear(x, *g), q8.linear(x, *u)
    want = qwen.silu_mul(gv, uv)
    tol = 2e-6 * (1.1 * bound(x, g) * np.abs(uv) + np.abs(gv) * bound(x, u)) + 1e-6 * np.abs(want) + 1e-30
    assert (np.abs(got - want) <= tol).all()


def test_wide_dynamic_range(env):
    """Activations spread over 2^-40 .. 2^40 with full 24-bit mantissas: the three bf16
    pieces must carry every bit, or the error would reach 2^-8 of the terms."""
    torch, ops = env
    rng = np.random.default_rng(12)
    m, n, k = 64, 256, 512
    x = (rng.standard_normal((m, k)) * np.exp2(rng.integers(-40, 41, (m, k)))).astype(np.float32)
    w = rand_q8(rng, n, k)
    got = ops.linear_q8(dev(torch, x), dev(torch, w[0]), dev(torch, w[1])).cpu().numpy()
    check(got, q8.linear(x, *w), bound(x, w))


def test_deterministic_and_distinct_from_cuda_cores(env):
    """k split over a cluster of CTAs (a few tiles): repeated calls are bit-identical, and the
    CUDA-core kernel's other summation order gives other roundings."""
    torch, ops = env
    rng = np.random.default_rng(9)
    x = dev(torch, rng.standard_normal((32, 4864), dtype=np.float32))
    qo, so = rand_q8(rng, 512, 4864)
    tq, ts = dev(torch, qo), dev(torch, so)
    outs = [ops.linear_q8(x, tq, ts).cpu() for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    ops.q8_tensor_cores(False)
    try:
        other = ops.linear_q8(x, tq, ts).cpu()
    finally:
        ops.q8_tensor_cores("always")
    assert not torch.equal(outs[0], other)


def test_switch_round_trips(env):
    torch, ops = env
    assert ops.q8_tensor_cores() == 2
    assert ops.q8_tensor_cores(False) == 2
    assert ops.q8_tensor_cores() == 0
    assert ops.q8_tensor_cores(True) == 0
    assert ops.q8_tensor_cores() == 1
    assert ops.q8_tensor_cores("always") == 1


def test_default_mode_routes_by_size(env):
    """The default setting sends a small product at up to 64 rows (k <= 1024, at most 1.25 M
    weights) to the CUDA-core kernel and a longer k to the tcgen05 kernel: bit-identical to
    the kernel forced for each (the two round differently, so the route is visible)."""
    torch, ops = env

    def run(mode, m, n, k):
        x = dev(torch, np.random.default_rng(m + n + k).standard_normal((m, k), dtype=np.float32))
        qo, so = rand_q8(np.random.default_rng(n * k), n, k)
        ops.q8_tensor_cores(mode)
        try:
            return ops.linear_q8(x, dev(torch, qo), dev(torch, so)).cpu()
        finally:
            ops.q8_tensor_cores("always")

    for m, n, k, small in ((32, 512, 512, True), (64, 2048, 512, True), (32, 512, 2048, False), (16, 4096, 512, False)):
        auto, cc, tc = run(1, m, n, k), run(False, m, n, k), run("always", m, n, k)
        assert not torch.equal(cc, tc), (m, n, k)
        assert torch.equal(auto, cc if small else tc), (m, n, k, small)


@pytest.mark.parametrize("tc", [True, False], ids=["tcgen05", "cuda_cores"])
def test_rope_pair_both_kernels(env, tc):
    """The Qwen2 q/k/v pair (bias, RoPE, q out, K^T scatter, V copy) at 16+ rows on either
    kernel against the oracle: heads of d 64 (two per 128-row tile) and d 128 (one), single
    tokens of 16 sequences (k split over a cluster) and 60- and 64-token chunks."""
    torch, ops = env
    from tests.test_gpu_llm_step import run_qkv
    ops.q8_tensor_cores("always" if tc else False)
    try:
        run_qkv(torch, ops, B=16, H=4, Hkv=2, d=64, n_ctx=32, chunks=[1, 1], seed=4)
        run_qkv(torch, ops, B=8, H=14, Hkv=2, d=64, n_ctx=128, chunks=[60, 1], seed=5)
        run_qkv(torch, ops, B=4, H=14, Hkv=2, d=128, n_ctx=128, chunks=[64, 1], seed=6, bias=False)
    finally:
        ops.q8_tensor_cores("always")
