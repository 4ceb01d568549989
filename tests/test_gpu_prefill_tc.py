"""Qwen2 prefill on the tf32 tensor-core kernel (csrc/attn_prefill_tc.cu) against the CPU
oracle (oracle/attention.py, src/ops.zig:562-590 with kt_stride), through zwg_attention_dev
with the context's math mode set to "tf32".

Shapes follow the Qwen2 attention call (src/llm.zig:178-202): q [n_q][n_head*d] after RoPE,
cache_kt [n_head_kv][d][n_ctx], cache_v [n_ctx][n_head_kv*d], prompt chunks of up to 256
queries (src/llm.zig:257-266), head h reading kv head h / (n_head / n_head_kv). The
tensor cores read the f32 operands as tf32 (10-bit mantissa), so the tolerance is the
north-star one, max-abs 2e-3 with rel 1e-3, not the f32 kernels' 1e-4. Each case also
checks from the CUDA activity trace that the tensor-core kernel is the one that ran.
"""
import numpy as np
import pytest

from oracle import attention as A
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu

TC_ATOL, TC_RTOL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    ops.set_math("tf32")
    yield torch, ops
    ops.set_math("f32")


def kernels_run(torch, fn):
    """Names of the events of one profiled call of fn. The activity trace occasionally comes
    back with the launch call but without the kernel's own record; the call (which only
    rewrites its output) is then profiled again, up to three times."""
    from torch.autograd import DeviceType
    from torch.profiler import ProfilerActivity, profile
    names = []
    for _ in range(3):
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        events = list(prof.events())
        names = [e.name for e in events]
        if any(e.device_type == DeviceType.CUDA for e in events):
            break
    return names


CASES = [
    # B, H, Hkv, d, n_ctx, n_past, n_q, causal
    (2, 14, 2, 64, 2048, 0, 256, True),       # Qwen2.5-0.5B, first prompt chunk
    (2, 14, 2, 64, 2048, 1792, 208, True),    # 0.5B, last chunk of a 2000-token prompt
    (2, 12, 2, 128, 2560, 1024, 256, True),   # Qwen2.5-1.5B, a middle chunk
    (3, 12, 2, 128, 2560, 1792, 208, True),   # 1.5B, last chunk
    (1, 14, 2, 64, 64, 20, 5, True),          # 5 queries x 7 heads: one partial tile
    (2, 16, 2, 128, 1024, 500, 77, True),     # group 8: 16 queries per tile, 128 rows
    (2, 4, 4, 64, 512, 0, 150, False),        # MHA, not causal, n_kv 150
    (1, 24, 2, 64, 768, 333, 100, True),      # group 12: 10 queries per tile, 120 rows
    # more items than CTAs (one per SM): each CTA runs several query tiles in a row, the
    # item-to-item hand-over of Q, the score buffers, O and the PV barriers
    (16, 14, 2, 64, 2048, 1792, 208, True),   # 0.5B last chunk, 384 items
    (16, 12, 2, 128, 2048, 1792, 208, True),  # 1.5B last chunk, 320 items
]


@pytest.mark.parametrize("B,H,Hkv,d,n_ctx,n_past,n_q,causal", CASES)
def test_prefill_tf32_matches_oracle(env, B, H, Hkv, d, n_ctx, n_past, n_q, causal):
    torch, ops = env
    rng = np.random.default_rng(1000 + n_past + n_q + d)
    n_kv = n_past + n_q
    kvw = Hkv * d
    q = rng.standard_normal((B, n_q, H * d), dtype=np.float32)
    kt = rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32)
    v = rng.standard_normal((B, n_ctx, kvw), dtype=np.float32)
    sh = ops.AttnShape(n_q, n_kv, H, Hkv, d, H * d, kvw, H * d, causal, n_ctx)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.full_like(tq, float("nan"))
    names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B))
    assert any("prefill_tc_kernel" in n for n in names), names
    got = out.cpu().numpy()
    sho = A.AttnShape(n_q, n_kv, H, Hkv, d, H * d, kvw, H * d, causal, n_ctx)
    for b in range(B):
        want = A.attention_ex(q[b].reshape(-1), kt[b].reshape(-1), v[b].reshape(-1), sho)
        np.testing.assert_allclose(got[b].reshape(-1), want, atol=TC_ATOL, rtol=TC_RTOL)


# d = 64 launches with enough items run two query tiles per item (a K/V tile feeds both, one
# softmax warpgroup each) when that form needs fewer waves of items by its weight (a paired
# item ~1.74 single ones) on 148 SMs; these shapes are chosen to take it: an even and an odd
# number of query tiles (the last pair's second tile past the end), several items per CTA,
# and a non-causal MHA launch.
PAIRED = [
    # B, H, Hkv, d, n_ctx, n_past, n_q, causal
    (16, 14, 2, 64, 2048, 1856, 144, True),   # 8 query tiles: 256 tiles, 128 pairs
    (16, 14, 2, 64, 1024, 900, 120, True),    # 7 query tiles: 224 tiles, 128 pairs
    (16, 14, 2, 64, 2048, 0, 256, True),      # first chunk: 480 tiles, 256 pairs
    (64, 4, 4, 64, 512, 0, 150, False),       # MHA, not causal: 512 tiles, 256 pairs
]


@pytest.mark.parametrize("B,H,Hkv,d,n_ctx,n_past,n_q,causal", PAIRED)
def test_prefill_tf32_two_tiles_per_item(env, B, H, Hkv, d, n_ctx, n_past, n_q, causal):
    torch, ops = env
    import re
    rng = np.random.default_rng(2000 + n_past + n_q + B)
    n_kv = n_past + n_q
    kvw = Hkv * d
    q = rng.standard_normal((B, n_q, H * d), dtype=np.float32)
    kt = rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32)
    v = rng.standard_normal((B, n_ctx, kvw), dtype=np.float32)
    sh = ops.AttnShape(n_q, n_kv, H, Hkv, d, H * d, kvw, H * d, causal, n_ctx)
    dev = torch.device("cuda:0")
    if torch.cuda.get_device_properties(dev).multi_processor_count != 148:
        pytest.skip("the shapes are chosen for 148 SMs")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.full_like(tq, float("nan"))
    names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B))
    assert any(re.search(r"prefill_tc_kernel<64, ?2>", n) for n in names), names
    got = out.cpu().numpy()
    sho = A.AttnShape(n_q, n_kv, H, Hkv, d, H * d, kvw, H * d, causal, n_ctx)
    for b in range(B):
        want = A.attention_ex(q[b].reshape(-1), kt[b].reshape(-1), v[b].reshape(-1), sho)
        np.testing.assert_allclose(got[b].reshape(-1), want, atol=TC_ATOL, rtol=TC_RTOL)


def test_prefill_tf32_rescale_path_two_tiles(env):
    """The rescale test's key growth with enough sequences for the paired form (20 x 2
    (sequence, kv head) pairs x 13 query tiles: 520 tiles, 280 pairs)."""
    torch, ops = env
    import re
    rng = np.random.default_rng(77)
    B, H, Hkv, d, n_ctx, n_past, n_q = 20, 12, 2, 64, 2048, 1744, 256
    n_kv = n_past + n_q
    slope = 0.5 + rng.random((B, n_q, 1), dtype=np.float32)
    q = (slope + 0.1 * rng.standard_normal((B, n_q, H * d), dtype=np.float32)).astype(np.float32)
    pos = np.arange(n_ctx, dtype=np.float32)
    kt = (0.2 * pos / 64 + 0.1 * rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32)).astype(np.float32)
    v = rng.standard_normal((B, n_ctx, Hkv * d), dtype=np.float32)
    sh = ops.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    dev = torch.device("cuda:0")
    if torch.cuda.get_device_properties(dev).multi_processor_count != 148:
        pytest.skip("the shape is chosen for 148 SMs")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.full_like(tq, float("nan"))
    names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B))
    assert any(re.search(r"prefill_tc_kernel<64, ?2>", n) for n in names), names
    sho = A.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    got = out.cpu().numpy()
    for b in (0, 7, 19):
        want = A.attention_ex(q[b].reshape(-1), kt[b].reshape(-1), v[b].reshape(-1), sho)
        np.testing.assert_allclose(got[b].reshape(-1), want, atol=TC_ATOL, rtol=TC_RTOL)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_tf32_rescale_path(env, d):
    """Keys scaled up with their position make the scores grow tile by tile, so the running
    max rises by more than 2^8 several times and the O-rescale branch runs (in some rows of
    a warp and not in others: each query row has its own slope)."""
    torch, ops = env
    rng = np.random.default_rng(41 + d)
    B, H, Hkv, n_ctx, n_past, n_q = 1, 12, 2, 2048, 1744, 256
    n_kv = n_past + n_q
    slope = 0.5 + rng.random((B, n_q, 1), dtype=np.float32)
    q = (slope + 0.1 * rng.standard_normal((B, n_q, H * d), dtype=np.float32)).astype(np.float32)
    pos = np.arange(n_ctx, dtype=np.float32)
    kt = (0.2 * pos / 64 * (64 / d) + 0.1 * rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32))
    kt = kt.astype(np.float32)
    v = rng.standard_normal((B, n_ctx, Hkv * d), dtype=np.float32)
    sh = ops.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.full_like(tq, float("nan"))
    names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B))
    assert any("prefill_tc_kernel" in n for n in names)
    sho = A.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    want = A.attention_ex(q[0].reshape(-1), kt[0].reshape(-1), v[0].reshape(-1), sho)
    np.testing.assert_allclose(out.cpu().numpy().reshape(-1), want, atol=TC_ATOL, rtol=TC_RTOL)


def test_prefill_tf32_strided_rows_and_batch(env):
    """Padded rows (q/out stride > n_head*d, kv stride > n_head_kv*d) and batch strides
    larger than one item: only the head columns of each output row are written."""
    torch, ops = env
    rng = np.random.default_rng(77)
    B, H, Hkv, d, n_ctx, n_q, n_kv = 2, 14, 2, 64, 1024, 96, 700
    qs, kvs, os_ = H * d + 64, Hkv * d + 32, H * d + 128
    q = rng.standard_normal((B, n_q + 3, qs), dtype=np.float32)
    kt = rng.standard_normal((B, Hkv, d, n_ctx + 64), dtype=np.float32)
    v = rng.standard_normal((B, n_ctx + 8, kvs), dtype=np.float32)
    sh = ops.AttnShape(n_q, n_kv, H, Hkv, d, qs, kvs, os_, True, n_ctx + 64)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.full((B, n_q + 1, os_), 7.0, device=dev)
    strides = (q[0].size, kt[0].size, v[0].size, out[0].numel())
    names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B, batch_strides=strides))
    assert any("prefill_tc_kernel" in n for n in names)
    got = out.cpu().numpy()
    sho = A.AttnShape(n_q, n_kv, H, Hkv, d, qs, kvs, os_, True, n_ctx + 64)
    for b in range(B):
        want = A.attention_ex(q[b].reshape(-1), kt[b].reshape(-1), v[b].reshape(-1), sho)
        want = want.reshape(n_q, os_)
        np.testing.assert_allclose(got[b, :n_q, :H * d], want[:, :H * d], atol=TC_ATOL, rtol=TC_RTOL)
        assert np.all(got[b, :, H * d:] == 7.0)   # padding columns untouched
        assert np.all(got[b, n_q:] == 7.0)        # rows past n_q untouched


def test_f32_mode_keeps_the_f32_kernel(env):
    """With the math mode back at "f32" the same call runs the f32 tiled kernel."""
    torch, ops = env
    rng = np.random.default_rng(3)
    B, H, Hkv, d, n_ctx, n_q, n_kv = 1, 14, 2, 64, 512, 64, 300
    q = rng.standard_normal((B, n_q, H * d), dtype=np.float32)
    kt = rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32)
    v = rng.standard_normal((B, n_ctx, Hkv * d), dtype=np.float32)
    sh = ops.AttnShape(n_q, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.empty_like(tq)
    ops.set_math("f32")
    try:
        names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B))
    finally:
        ops.set_math("tf32")
    assert not any("prefill_tc_kernel" in n for n in names)
    assert any("flash_f32_kernel" in n for n in names)
