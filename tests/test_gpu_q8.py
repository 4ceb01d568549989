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
    """m >= 16 runs every full chunk of 8 x rows in one launch (grid.y) and the rest in another."""
    torch, ops = env
    check_linear(torch, ops, m, n, k, bias=(m % 2 == 1), seed=m * 100 + n + k)


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
