"""The batched host-pointer entry point (zwg_attention_batch_host: ops.attentionEx over
n_batch items in host memory, src/ops.zig:562-590) against the CPU oracle
(oracle/attention.py), through the C ABI.

The call stages the items through a ring of device slots in chunks that grow 1, 2, 4, ...
at the start and shrink the same way at the end, and copies a chunk's q, k, v (and its
output) in one copy each when the items lie back to back on the host, else item by item
(and then only the head columns of each output row). Covered: batch sizes that give no
ramp, a short one and a full one; items back to back; gaps between items with rows wider
than the heads (the gaps and the extra columns of `out` are left as they were); and the
bf16 tensor-core route of the math mode "bf16" (the encoder-shaped calls).
"""
import ctypes

import numpy as np
import pytest

from oracle import attention as A
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu

F32_ATOL = 1e-4
BF16_ATOL, BF16_RTOL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def ops():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    from zwhisper_b200 import ops as o
    return o


def rnd(rng, n):
    return (rng.random(n, dtype=np.float32) - 0.5).astype(np.float32)


@pytest.mark.parametrize("nb", [1, 2, 5, 13, 40])
def test_back_to_back_items(ops, nb):
    rng = np.random.default_rng(100 + nb)
    n_q, n_kv, H, Hkv, d = 33, 70, 4, 2, 64
    sh_o = A.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True)
    sh = ops.AttnShape(**sh_o.__dict__)
    nq, nk, nv, no = sh.extents()
    q, k, v = rnd(rng, nq * nb), rnd(rng, nk * nb), rnd(rng, nv * nb)
    got = ops.attention_batch_host(q, k, v, sh, nb)
    for i in range(nb):
        want = A.attention_ex(q[i * nq:(i + 1) * nq], k[i * nk:(i + 1) * nk], v[i * nv:(i + 1) * nv], sh_o)
        np.testing.assert_allclose(got[i * no:(i + 1) * no], want, atol=F32_ATOL, rtol=0)


@pytest.mark.parametrize("nb", [3, 13])
def test_gaps_between_items_and_wide_rows(ops, nb):
    """Batch strides past each item's extent and rows wider than the heads: the copies go
    item by item (2-D for the output) and every float outside the head columns of `out`
    keeps its value."""
    from zwhisper_b200 import _lib
    rng = np.random.default_rng(200 + nb)
    n_q, n_kv, H, d = 21, 45, 2, 64
    sh_o = A.AttnShape(n_q, n_kv, H, H, d, H * d + 16, H * d + 32, H * d + 8, False)
    sh = ops.AttnShape(**sh_o.__dict__)
    nq, nk, nv, no = sh.extents()
    qbs, kbs, vbs, obs = nq + 40, nk + 24, nv + 8, no + 36
    q, k, v = rnd(rng, qbs * nb), rnd(rng, kbs * nb), rnd(rng, vbs * nb)
    out = np.full(obs * nb, 7.0, np.float32)
    _lib.ensure_init(0)
    lib = _lib.load()
    c = sh.to_c()
    b = _lib.BatchC(nb, qbs, kbs, vbs, obs)
    _lib.check(lib.zwg_attention_batch_host(ctypes.byref(c), ctypes.byref(b), q.ctypes.data, k.ctypes.data,
                                            v.ctypes.data, out.ctypes.data))
    for i in range(nb):
        want = A.attention_ex(q[i * qbs:i * qbs + nq], k[i * kbs:i * kbs + nk], v[i * vbs:i * vbs + nv], sh_o,
                              out=np.full(no, 7.0, np.float32))
        np.testing.assert_allclose(out[i * obs:i * obs + no], want, atol=F32_ATOL, rtol=0)
        assert (out[i * obs + no:(i + 1) * obs] == 7.0).all()


def test_bf16_route_matches_oracle(ops):
    """Math mode "bf16": Whisper tiny.en-shaped encoder calls (1500 frames, 6 heads of 64)
    for 5 windows back to back run the bf16 tcgen05 kernel; checked against the float64
    oracle on the same bf16-rounded inputs."""
    import torch
    rng = np.random.default_rng(7)
    nb, n_ctx, H = 5, 1500, 6
    ns = H * 64
    sh = ops.mha_shape(n_ctx, n_ctx, ns, H, False)
    q, k, v = (rng.standard_normal(nb * n_ctx * ns, dtype=np.float32) for _ in range(3))
    ops.set_math("bf16")
    try:
        got = ops.attention_batch_host(q, k, v, sh, nb)
    finally:
        ops.set_math("f32")

    def bf16(x):
        return torch.from_numpy(x).to(torch.bfloat16).float().numpy()

    def heads(x):
        return x.reshape(nb, n_ctx, H, 64).transpose(0, 2, 1, 3)

    want = A.attention_batched(heads(bf16(q)), heads(bf16(k)), heads(bf16(v)), causal=False)
    want = want.transpose(0, 2, 1, 3).reshape(-1)
    np.testing.assert_allclose(got, want, atol=BF16_ATOL, rtol=BF16_RTOL)
