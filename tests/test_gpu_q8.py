"""The Q8 kernels (csrc/q8.cu) against the oracle (oracle/q8.py, src/gemm.zig:188-351,
src/ops.zig:280-306) through the C ABI: zwg_q8_quantize must reproduce Q8.quantize bit for
bit (int8 values and f32 scales); zwg_linear_q8 is f32 arithmetic in another summation
order, held to a relative error of 2e-6 of the sum of |x . w| terms (about 16 f32 ulps)."""
import numpy as np
import pytest

from oracle import q8
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    return torch, ops


@pytest.mark.parametrize("n,k", [(7, 64), (512, 512), (256, 1536), (33, 8960)])
def test_quantize_bit_exact(env, n, k):
    torch, ops = env
    rng = np.random.default_rng(n + k)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    w[0, :32] = 0.0           # an all-zero block: scale 0, q 0
    w[1, 5] = 3.0             # a block with one large weight
    qo, so = q8.quantize(w)
    q, s = ops.quantize_q8(torch.from_numpy(w).cuda())
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))


def check_linear(torch, ops, m, n, k, bias, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    b = rng.standard_normal(n, dtype=np.float32) if bias else None
    qo, so = q8.quantize(w)
    want = q8.linear(x, qo, so, b)
    dev = torch.device("cuda:0")
    tq, ts = torch.from_numpy(qo).to(dev), torch.from_numpy(so).to(dev)
    tb = torch.from_numpy(b).to(dev) if bias else None
    got = ops.linear_q8(torch.from_numpy(x).to(dev), tq, ts, tb).cpu().numpy()
    # error scale: the sum of |terms| of each output
    mag = np.abs(x).astype(np.float64) @ np.abs(q8.dequant(qo, so)).astype(np.float64).T
    if bias:
        mag = mag + np.abs(b)[None]
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert (err <= 2e-6 * mag + 1e-30).all(), float((err / (mag + 1e-30)).max())


@pytest.mark.parametrize("m", [1, 2, 3, 8, 13, 37])
@pytest.mark.parametrize("n,k", [(1, 32), (7, 64), (512, 512), (1536, 1536), (101, 8960)])
def test_linear_matches_oracle(env, m, n, k):
    """Up to 15 rows run in chunks of 8 rows of x; 16 or more (37 here) the register-tiled
    product."""
    torch, ops = env
    check_linear(torch, ops, m, n, k, bias=(m % 2 == 1), seed=m * 100 + n + k)


@pytest.mark.parametrize("m,n,k", [(32, 4096, 512), (64, 1536, 8960), (64, 2048, 1536), (16, 100, 96),
                                   (32, 8192, 512), (64, 8960, 1536), (200, 2048, 256)])
def test_linear_many_rows(env, m, n, k):
    """16 or more rows run the register-tiled product: shapes with at least 64 tiles of 32 or
    64 rows x 128 columns on those (8192 or 8960 columns, 200 rows with a partial row tile),
    the others on 32 x 64 tiles with k split over a cluster of CTAs and reduced through
    distributed shared memory (100 columns: a partial tile)."""
    torch, ops = env
    check_linear(torch, ops, m, n, k, bias=(n % 2 == 0), seed=m + n + k)


def test_linear_many_rows_deterministic(env):
    """The split-K reduction sums the partial tiles in a fixed order: repeated calls are
    bit-identical."""
    torch, ops = env
    rng = np.random.default_rng(9)
    dev = torch.device("cuda:0")
    x = torch.from_numpy(rng.standard_normal((32, 512), dtype=np.float32)).to(dev)
    qo, so = q8.quantize((rng.standard_normal((512, 512), dtype=np.float32) * 0.02).astype(np.float32))
    tq, ts = torch.from_numpy(qo).to(dev), torch.from_numpy(so).to(dev)
    outs = [ops.linear_q8(x, tq, ts, None).cpu() for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_linear_set_audio_shape(env):
    """1500 rows of x, the Whisper decoder's cross K/V projection (src/decoder.zig:154-155)."""
    torch, ops = env
    check_linear(torch, ops, 1500, 96, 128, bias=True, seed=5)


def test_whisper_logits_matvec_shape(env):
    """The decoder's logits product (src/decoder.zig:412-413): 51864 x 512, one token."""
    torch, ops = env
    check_linear(torch, ops, 1, 51864, 512, bias=False, seed=1)


def test_rejects_bad_k(env):
    torch, ops = env
    from zwhisper_b200 import _lib
    x = torch.zeros(1, 48, device="cuda:0")
    q = torch.zeros(4, 48, dtype=torch.int8, device="cuda:0")
    s = torch.zeros(4 * 48 // 32 + 1, device="cuda:0")
    with pytest.raises(_lib.ZwgError, match="multiple of 32"):
        _lib.check(_lib.load().zwg_linear_q8(x.data_ptr(), 1, 48, q.data_ptr(), s.data_ptr(), None, 4,
                                             x.data_ptr(), None))
