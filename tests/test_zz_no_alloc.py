"""zwg_attention_dev_noalloc: the decode attention entry point that allocates nothing.

Some callers cannot call cudaMalloc (an embedding that only has this C ABI and no CUDA
allocator bindings, or a streaming decode thread that must not stall on an allocation that
synchronizes the device). For them the split-K partials live in a fixed 4 MiB device array
inside the library. These checks call it through the C ABI:
  - against the CPU oracle (oracle/attention.py, the restatement of ops.attentionEx) at the
    f32 tolerance of the other decode tests, over both key layouts, d 32/64/128, GQA groups
    1/2/4, several query rows with the causal mask (including a split whose key chunk is
    fully masked for some rows), key counts that are not multiples of the tile, and no keys;
  - twice in a row (the second call starts from what the first left in the shared array)
    against the ordinary entry point, zwg_attention_dev with caller workspace;
  - for the rejections: a call needing more than the array holds, and (no GPU needed) a
    shape the shared checks refuse before any CUDA call.
The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

from oracle import attention as OA
from tests.conftest import has_gpu

F32_ATOL = 1e-4


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import _lib, ops
    return torch, _lib, ops


def noalloc_call(torch, _lib, sh, n_batch, q, k, v, out):
    lib = _lib.load()
    c = sh.to_c()
    b = _lib.BatchC(n_batch, q.numel() // n_batch, k.numel() // n_batch, v.numel() // n_batch,
                    out.numel() // n_batch)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.zwg_attention_dev_noalloc(ctypes.byref(c), ctypes.byref(b), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                       out.data_ptr(), stream)
    _lib.check(rc)


# (kt layout, d, group, n_q, causal, n_kv): every shape keeps n_q * group <= 8 query rows per
# kv head, the decode limit; 3001 and 2049 keys take several splits (chunks of 512 keys for
# the K^T layout, 128 for rows), and 2049 with n_q 2 leaves a last chunk of one key that row
# 0 of each group cannot see.
ORACLE_CASES = [
    (True, 128, 6, 1, True, 3001),
    (True, 64, 7, 1, True, 2049),
    (True, 64, 4, 2, True, 2049),
    (True, 32, 2, 4, True, 1000),
    (True, 128, 1, 1, False, 77),
    (True, 32, 4, 2, False, 3001),
    (False, 64, 1, 1, False, 1500),
    (False, 64, 1, 4, True, 225),
    (False, 32, 2, 2, True, 3001),
    (False, 128, 4, 2, True, 2049),
    (False, 128, 2, 1, False, 1),
    (False, 64, 1, 1, False, 0),
    (True, 64, 2, 1, False, 0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("kt,d,group,n_q,causal,n_kv", ORACLE_CASES)
def test_matches_oracle(env, kt, d, group, n_q, causal, n_kv):
    torch, _lib, ops = env
    rng = np.random.default_rng(1000 * d + 10 * group + n_q + n_kv)
    B, Hkv = 2, 2
    H = Hkv * group
    n_ctx = (max(n_kv, 1) + 3) // 4 * 4 + 8 if kt else None
    sh = ops.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, causal, n_ctx)
    q = rng.standard_normal((B, n_q * H * d), dtype=np.float32)
    if kt:
        k = rng.standard_normal((B, Hkv * d * n_ctx), dtype=np.float32)
        v = rng.standard_normal((B, n_ctx * Hkv * d), dtype=np.float32)
    else:
        k = rng.standard_normal((B, max(n_kv, 1) * Hkv * d), dtype=np.float32)
        v = rng.standard_normal((B, max(n_kv, 1) * Hkv * d), dtype=np.float32)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    got = torch.full_like(tq, float("nan"))
    noalloc_call(torch, _lib, sh, B, tq, tk, tv, got)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    osh = OA.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, causal, n_ctx)
    for b in range(B):
        want = OA.attention_ex(q[b], k[b], v[b], osh)
        np.testing.assert_allclose(got[b], want[:n_q * H * d], atol=F32_ATOL, rtol=0)


@pytest.mark.gpu
def test_two_calls_in_a_row_match_workspace_entry_point(env):
    torch, _lib, ops = env
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    cases = []
    # Qwen2.5-1.5B-shaped decode over the transposed key cache
    B, H, Hkv, d, n_ctx, n_kv = 8, 12, 2, 128, 2560, 2001
    cases.append((ops.AttnShape(1, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx), B,
                  torch.randn(B, H * d, generator=g, device=dev),
                  torch.randn(B, Hkv, d, n_ctx, generator=g, device=dev),
                  torch.randn(B, n_ctx, Hkv * d, generator=g, device=dev)))
    # Whisper base.en cross-attention step over 1500 keys
    B2, ns = 32, 512
    cases.append((ops.mha_shape(1, 1500, ns, 8, False), B2,
                  torch.randn(B2, 1, ns, generator=g, device=dev),
                  torch.randn(B2, 1500, ns, generator=g, device=dev),
                  torch.randn(B2, 1500, ns, generator=g, device=dev)))
    for sh, nb, q, k, v in cases:
        want = torch.empty_like(q)
        ops.attention_dev(q, k, v, sh, want, n_batch=nb)
        for _ in range(2):
            got = torch.full_like(q, float("nan"))
            noalloc_call(torch, _lib, sh, nb, q, k, v, got)
            torch.cuda.synchronize()
            np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), atol=F32_ATOL, rtol=0)


@pytest.mark.gpu
def test_rejects_calls_beyond_the_scratch_limit(env):
    torch, _lib, ops = env
    dev = torch.device("cuda:0")
    # 512 sequences x 2 kv heads x 6 rows x splits x 130 floats is far beyond 4 MiB
    B, H, Hkv, d, n_ctx, n_kv = 512, 12, 2, 128, 2048, 2048
    sh = ops.AttnShape(1, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    q = torch.zeros(B, H * d, device=dev)
    k = torch.zeros(1, device=dev)  # never read: the call must fail before launching
    out = torch.zeros_like(q)
    lib = _lib.load()
    c = sh.to_c()
    b = _lib.BatchC(B, H * d, Hkv * d * n_ctx, n_ctx * Hkv * d, H * d)
    rc = lib.zwg_attention_dev_noalloc(ctypes.byref(c), ctypes.byref(b), q.data_ptr(), k.data_ptr(), k.data_ptr(),
                                       out.data_ptr(), None)
    assert rc == _lib.ZWG_ERROR
    assert "4 MiB" in _lib.last_error()
    torch.cuda.synchronize()


def test_rejects_oversized_shapes_without_a_gpu():
    """The shape checks run before any CUDA call, so these need no device: keys beyond the
    2^30 the kernels index with 32-bit integers, and a missing shape."""
    from zwhisper_b200 import _lib, ops
    lib = _lib.load()
    sh = ops.AttnShape(1, (1 << 30) + 4, 12, 2, 128, 12 * 128, 2 * 128, 12 * 128, True, (1 << 30) + 8)
    c = sh.to_c()
    rc = lib.zwg_attention_dev_noalloc(ctypes.byref(c), None, None, None, None, None, None)
    assert rc == _lib.ZWG_ERROR
    assert "too long" in _lib.last_error()
    rc = lib.zwg_attention_dev_noalloc(None, None, None, None, None, None, None)
    assert rc == _lib.ZWG_ERROR
    assert "null shape" in _lib.last_error()
