"""zwg_attention_dev_noalloc: the decode attention entry point that allocates nothing.

Some callers cannot call cudaMalloc (an embedding that only has this C ABI and no CUDA
allocator bindings, or a streaming decode thread that must not stall on an allocation that
synchronizes the device). For them the split-K partials live in a fixed 4 MiB device array
inside the library. These checks call it through the C ABI twice in a row (the second call
starts from what the first left in the shared array) and compare each result with the
ordinary entry point, zwg_attention_dev with caller workspace, at the f32 tolerance the
other decode tests use. The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu

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


def test_two_calls_match_workspace_entry_point(env):
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
    B2, ns = 16, 512
    cases.append((ops.mha_shape(1, 1500, ns, 8, False), B2,
                  torch.randn(B2, 1, ns, generator=g, device=dev),
                  torch.randn(B2, 1500, ns, generator=g, device=dev),
                  torch.randn(B2, 1500, ns, generator=g, device=dev)))
    for sh, nb, q, k, v in cases:
        want = torch.empty_like(q)
        ops.attention_dev(q, k, v, sh, want, n_batch=nb)
        got = torch.full_like(q, float("nan"))
        noalloc_call(torch, _lib, sh, nb, q, k, v, got)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), atol=F32_ATOL, rtol=0)


def test_same_call_twice_in_a_row(env):
    torch, _lib, ops = env
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    B, ns = 32, 512
    sh = ops.mha_shape(1, 1500, ns, 8, False)
    q = torch.randn(B, 1, ns, generator=g, device=dev)
    k = torch.randn(B, 1500, ns, generator=g, device=dev)
    v = torch.randn(B, 1500, ns, generator=g, device=dev)
    want = torch.empty_like(q)
    ops.attention_dev(q, k, v, sh, want, n_batch=B)
    for _ in range(2):
        got = torch.full_like(q, float("nan"))
        noalloc_call(torch, _lib, sh, B, q, k, v, got)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), atol=F32_ATOL, rtol=0)


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
