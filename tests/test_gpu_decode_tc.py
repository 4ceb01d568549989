"""Qwen2 decode on the tf32 tensor-core kernel (csrc/attn_decode_tc.cu) against the CPU
oracle (oracle/attention.py, src/ops.zig:562-590 with kt_stride), through zwg_attention_dev
with the context's math mode set to "tf32".

Shapes follow the Qwen2 decode call (src/llm.zig:178-202 with n = 1): q [1][n_head*d] after
RoPE, cache_kt [n_head_kv][d][n_ctx], cache_v [n_ctx][n_head_kv*d], head h reading kv head
h / (n_head / n_head_kv). The cases cover one segment cut into 16 pieces (the merge by the
last CTA), whole segments per CTA (64 sequences), 9 pieces at d = 64, key counts that are
not multiples of the 64-key tile, a single short tile, and groups of 1, 6, 7 and 8. The
tensor cores read the f32 operands as tf32, so the tolerance is the north-star one,
max-abs 2e-3 with rel 1e-3. Each case checks from the CUDA activity trace that the
tensor-core kernel ran."""
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
    # B, H, Hkv, d, n_ctx, n_kv
    (1, 12, 2, 128, 2560, 2256),   # Qwen2.5-1.5B, one sequence: 16 pieces per segment
    (64, 12, 2, 128, 2560, 2256),  # configs[4]'s batch: whole segments
    (16, 14, 2, 64, 2560, 2128),   # configs[3]: Qwen2.5-0.5B, 9 pieces of ~4 tiles
    (3, 14, 2, 64, 768, 700),      # 700 keys: a partial last tile
    (2, 16, 2, 128, 256, 5),       # 5 keys: one short tile; group 8
    (2, 4, 4, 64, 512, 301),       # group 1
]


def run_case(torch, ops, B, H, Hkv, d, n_ctx, n_kv, seed):
    rng = np.random.default_rng(seed)
    kvw = Hkv * d
    q = rng.standard_normal((B, 1, H * d), dtype=np.float32)
    kt = rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32)
    v = rng.standard_normal((B, n_ctx, kvw), dtype=np.float32)
    sh = ops.AttnShape(1, n_kv, H, Hkv, d, H * d, kvw, H * d, True, n_ctx)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.full_like(tq, float("nan"))
    names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B))
    assert any("decode_tc_kernel" in n for n in names), names
    got = out.cpu().numpy()
    sho = A.AttnShape(1, n_kv, H, Hkv, d, H * d, kvw, H * d, True, n_ctx)
    for b in range(B):
        want = A.attention_ex(q[b].reshape(-1), kt[b].reshape(-1), v[b].reshape(-1), sho)
        np.testing.assert_allclose(got[b].reshape(-1), want, atol=TC_ATOL, rtol=TC_RTOL)


@pytest.mark.parametrize("B,H,Hkv,d,n_ctx,n_kv", CASES)
def test_decode_tf32_matches_oracle(env, B, H, Hkv, d, n_ctx, n_kv):
    torch, ops = env
    run_case(torch, ops, B, H, Hkv, d, n_ctx, n_kv, seed=2000 + B + n_kv + d)


@pytest.mark.parametrize("B,H,d", [(40, 12, 128), (1, 14, 64)])
def test_decode_tf32_growing_scores(env, B, H, d):
    """Keys scaled up with their position make the scores grow tile by tile. With 40
    sequences every CTA holds a whole segment of 32 tiles, so the running max rises by more
    than 2^8 inside a CTA and the O-rescale branch runs; with one sequence the 16 pieces of
    a segment hold very different maxima, which the last CTA's merge scales together."""
    torch, ops = env
    rng = np.random.default_rng(43 + d + B)
    Hkv, n_ctx, n_kv = 2, 2048, 2000
    slope = 0.5 + rng.random((B, 1, 1), dtype=np.float32)
    q = (slope + 0.1 * rng.standard_normal((B, 1, H * d), dtype=np.float32)).astype(np.float32)
    pos = np.arange(n_ctx, dtype=np.float32)
    kt = (0.2 * pos / 64 * (64 / d) + 0.1 * rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32))
    kt = kt.astype(np.float32)
    v = rng.standard_normal((B, n_ctx, Hkv * d), dtype=np.float32)
    sh = ops.AttnShape(1, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    out = torch.full_like(tq, float("nan"))
    names = kernels_run(torch, lambda: ops.attention_dev(tq, tk, tv, sh, out, n_batch=B))
    assert any("decode_tc_kernel" in n for n in names), names
    sho = A.AttnShape(1, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    got = out.cpu().numpy()
    for b in range(B):
        want = A.attention_ex(q[b].reshape(-1), kt[b].reshape(-1), v[b].reshape(-1), sho)
        np.testing.assert_allclose(got[b].reshape(-1), want, atol=TC_ATOL, rtol=TC_RTOL)


def test_decode_tf32_repeated_calls(env):
    """The segment tickets are reset by the merging CTA: back-to-back calls on the same
    workspace give the same result."""
    torch, ops = env
    rng = np.random.default_rng(5)
    B, H, Hkv, d, n_ctx, n_kv = 2, 12, 2, 128, 1024, 1000
    q = rng.standard_normal((B, 1, H * d), dtype=np.float32)
    kt = rng.standard_normal((B, Hkv, d, n_ctx), dtype=np.float32)
    v = rng.standard_normal((B, n_ctx, Hkv * d), dtype=np.float32)
    sh = ops.AttnShape(1, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    dev = torch.device("cuda:0")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kt, v))
    ws = torch.empty(ops.attention_workspace_bytes(sh, B), dtype=torch.uint8, device=dev)
    outs = []
    for _ in range(3):
        out = torch.empty_like(tq)
        ops.attention_dev(tq, tk, tv, sh, out, n_batch=B, workspace=ws)
        outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    ops.sync()
