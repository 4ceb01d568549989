"""The Qwen2 decode step around the attention (include/zwgpu.h: zwg_rms_norm,
zwg_linear_q8_add, zwg_linear_q8_silu_mul, zwg_embed_q8, zwg_llm_greedy, zwg_llm_qkv_q8,
zwg_llm_layer_q8, zwg_llm_forward_q8) against the oracle (oracle/qwen.py, oracle/q8.py;
src/llm.zig:169-216, 268-321).

Tolerances: the embedding rows, the RoPE rotation of given values and the greedy choice are
exact; the projections are f32 sums in another order than the reference's (relative 2e-6 of
the sum of |terms|, as tests/test_gpu_q8.py); hidden states and logits after whole layers
are held to abs 1e-4 + rel 1e-4, well inside the hot path's max-abs 2e-3 / rel 1e-3; the
greedy tokens of a whole decode must be identical."""
import numpy as np
import pytest

from oracle import q8
from oracle import qwen
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu

STEP_ATOL = 1e-4
STEP_RTOL = 1e-4


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    ops.set_math("f32")
    return torch, ops


def dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    return t if dtype is None else t.to(dtype)


def rand_q8(rng, n, k):
    return q8.quantize((rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32))


def bound(x, qs):
    """Sum of |terms| of each output of x . W^T."""
    return np.abs(x).astype(np.float64) @ np.abs(q8.dequant(*qs)).astype(np.float64).T


@pytest.mark.parametrize("m,n", [(1, 896), (5, 1536), (3, 4)])
def test_rms_norm(env, m, n):
    torch, ops = env
    rng = np.random.default_rng(m * n)
    x = rng.standard_normal((m, n), dtype=np.float32)
    w = rng.standard_normal(n, dtype=np.float32)
    got = ops.rms_norm(dev(torch, x), dev(torch, w), 1e-6).cpu().numpy()
    np.testing.assert_allclose(got, qwen.rms_norm(x, w, 1e-6), rtol=2e-6, atol=1e-7)


def test_embed_bit_exact_and_bad_token(env):
    torch, ops = env
    from zwhisper_b200 import _lib
    rng = np.random.default_rng(5)
    q, s = rand_q8(rng, 300, 128)
    tq, ts = dev(torch, q), dev(torch, s)
    toks = np.array([7, 0, 299, 7], np.int32)
    got = ops.embed_q8(dev(torch, toks), tq, ts).cpu().numpy()
    assert np.array_equal(got, qwen.embed(q, s, toks))
    bad = ops.embed_q8(dev(torch, np.array([3, 300], np.int32)), tq, ts)
    with pytest.raises(_lib.ZwgError, match="device error"):
        ops.sync()
    assert np.array_equal(bad.cpu().numpy()[1], np.zeros(128, np.float32))
    ops.sync()  # the error word was cleared by the report


@pytest.mark.parametrize("m", [1, 2, 3, 8, 13])
@pytest.mark.parametrize("n,k", [(101, 256), (1536, 1536), (64, 8960)])
def test_linear_q8_add(env, m, n, k):
    torch, ops = env
    rng = np.random.default_rng(m + n + k)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rand_q8(rng, n, k)
    resid = rng.standard_normal((m, n), dtype=np.float32)
    out = dev(torch, resid)
    ops.linear_q8_add(dev(torch, x), dev(torch, w[0]), dev(torch, w[1]), out)
    want = (resid.astype(np.float64) + q8.linear(x, *w).astype(np.float64))
    err = np.abs(out.cpu().numpy() - want)
    assert (err <= 2e-6 * (bound(x, w) + np.abs(resid)) + 1e-30).all()


@pytest.mark.parametrize("m", [1, 2, 3, 8, 13, 16, 64])
@pytest.mark.parametrize("n,k", [(101, 256), (1000, 1536), (33, 896), (4096, 512)])
def test_linear_q8_silu_mul(env, m, n, k):
    torch, ops = env
    rng = np.random.default_rng(10 * m + n + k)
    x = rng.standard_normal((m, k), dtype=np.float32)
    g, u = rand_q8(rng, n, k), rand_q8(rng, n, k)
    got = ops.linear_q8_silu_mul(dev(torch, x), (dev(torch, g[0]), dev(torch, g[1])),
                                 (dev(torch, u[0]), dev(torch, u[1]))).cpu().numpy()
    gv, uv = q8.linear(x, *g), q8.linear(x, *u)
    want = qwen.silu_mul(gv, uv)
    # dot-product error (2e-6 of the |terms|) through silu' <= 1.1 and the product, plus exp's
    tol = 2e-6 * (1.1 * bound(x, g) * np.abs(uv) + np.abs(gv) * bound(x, u)) + 1e-6 * np.abs(want) + 1e-30
    assert (np.abs(got - want) <= tol).all()


def test_greedy_kernel(env):
    torch, ops = env
    rng = np.random.default_rng(6)
    m, V, steps = 5, 5000, 6
    logits = rng.standard_normal((m, V), dtype=np.float32)
    logits[1, 100] = logits[1, 200] = 9.0           # a tie: the first index wins
    logits[2, 0] = np.nan                           # NaN in column 0: the answer is 0
    logits[3, 50] = np.nan                          # NaN elsewhere never wins
    logits[3, 51] = 8.0
    recent = rng.integers(0, V, (m, steps)).astype(np.int32)
    recent[0, :4] = [7, 7, 7, 9]                    # repeats are penalized again
    logits[0, 7] = 9.5
    logits[0, 9] = 9.4
    logits[4, recent[4, 0]] = 20.0                  # outside the window: not penalized
    n_recent, window = 5, 3
    t_logits = dev(torch, logits)
    t_recent = dev(torch, recent)
    out = torch.full((m, steps + 1), -1, dtype=torch.int32, device="cuda:0")
    ops.llm_greedy(t_logits, t_recent, n_recent=n_recent, window=window, penalty=1.1, out=out[:, 2])
    got_l = t_logits.cpu().numpy()
    for i in range(m):
        row = logits[i].copy()
        want = qwen.greedy(row, recent[i, :n_recent], window=window, penalty=1.1)
        assert int(out[i, 2]) == want, i
        np.testing.assert_array_equal(got_l[i], row)
    assert (out[:, :2] == -1).all() and (out[:, 3:] == -1).all()  # only the given column is written


def run_qkv(torch, ops, B, H, Hkv, d, n_ctx, chunks, seed, bias=True):
    rng = np.random.default_rng(seed)
    ne = H * d
    st = ops.LlmState(1, B, H, Hkv, d, n_ctx, rope_base=1e6)
    m = qwen.make_model(seed, 1, 64, H, Hkv, d, 64, n_ctx, bias=bias)
    W = ops.LlmWeightsQ8(m["layers"], m["embd"], None, m["output_norm"], 1e-6)
    L = m["layers"][0]
    kt_o = [np.zeros(Hkv * d * n_ctx, np.float32) for _ in range(B)]
    v_o = [np.zeros(Hkv * d * n_ctx, np.float32) for _ in range(B)]
    n_past = 0
    for n in chunks:
        x = rng.standard_normal((B, n, ne), dtype=np.float32)
        got_q = st.qkv_q8(0, dev(torch, x), W, n_past).cpu().numpy()
        for b in range(B):
            q = q8.linear(x[b], *L["wq"], L["bq"])
            k = q8.linear(x[b], *L["wk"], L["bk"])
            v = q8.linear(x[b], *L["wv"], L["bv"])
            qr, _, _ = qwen.rope_and_append(q, k, v, kt_o[b], v_o[b], m["cos"], m["sin"], n_past, H, Hkv, d)
            np.testing.assert_allclose(got_q[b], qr, atol=2e-5, rtol=1e-5)
        n_past += n
    kt_t, v_t = st.cache_views(0)
    kt_g = kt_t.cpu().numpy().reshape(B, -1)
    v_g = v_t.cpu().numpy().reshape(B, n_ctx, -1)
    for b in range(B):
        # the K^T cache is zeroed at creation, so all of it compares; V rows past n_past are
        # never written or read
        np.testing.assert_allclose(kt_g[b], kt_o[b], atol=2e-5, rtol=1e-5)
        np.testing.assert_allclose(v_g[b, :n_past], v_o[b].reshape(n_ctx, -1)[:n_past], atol=2e-5, rtol=1e-5)
    st.close()


def test_qkv_q8_rope_append(env):
    torch, ops = env
    run_qkv(torch, ops, B=2, H=4, Hkv=2, d=64, n_ctx=64, chunks=[5, 1, 1], seed=1)


def test_qkv_q8_d128_many_rows(env):
    """d = 128 (Qwen2.5-1.5B heads) and 9 rows per call (chunks of 8 and 1)."""
    torch, ops = env
    run_qkv(torch, ops, B=3, H=6, Hkv=2, d=128, n_ctx=32, chunks=[3, 1], seed=2)
    run_qkv(torch, ops, B=1, H=6, Hkv=2, d=128, n_ctx=32, chunks=[9, 1], seed=3, bias=False)


def test_qkv_q8_many_rows_tiled(env):
    """16 or more rows per call run the pair on the tiled Q8 product: 16 sequences of one
    token (32 x 64 tiles), then chunks of 60 and 64 tokens whose 64 x 128 tiles span two heads
    (d 64) or one head (d 128); the next single-token call runs the 8-row path on the same
    caches."""
    torch, ops = env
    run_qkv(torch, ops, B=16, H=4, Hkv=2, d=64, n_ctx=32, chunks=[1, 1], seed=4)
    run_qkv(torch, ops, B=8, H=14, Hkv=2, d=64, n_ctx=128, chunks=[60, 1], seed=5)
    run_qkv(torch, ops, B=4, H=14, Hkv=2, d=128, n_ctx=128, chunks=[64, 1], seed=6, bias=False)


def device_model(ops, m):
    return ops.LlmWeightsQ8(m["layers"], m["embd"], None if m["output"] is m["embd"] else m["output"],
                            m["output_norm"], m["cfg"]["eps"])


def new_state(ops, m, B):
    c = m["cfg"]
    return ops.LlmState(c["n_layer"], B, c["n_head"], c["n_head_kv"], c["d"], c["n_ctx"], rope_base=c["rope_base"])


def test_layer_q8(env):
    torch, ops = env
    m = qwen.make_model(7, n_layer=1, n_vocab=100, n_head=4, n_head_kv=2, d=64, n_ff=512, n_ctx=32)
    B = 2
    W = device_model(ops, m)
    st = new_state(ops, m, B)
    caches = qwen.new_caches(m, B)
    rng = np.random.default_rng(8)
    n_past = 0
    for n in (6, 1):
        x = (rng.standard_normal((B, n, 256), dtype=np.float32) * np.float32(0.5)).astype(np.float32)
        got = st.layer_q8(0, W, dev(torch, x), n_past).cpu().numpy()
        c = m["cfg"]
        for b in range(B):
            xb = x[b].copy()
            qwen.layer_forward(xb, m["layers"][0], caches[b][0][0], caches[b][0][1], n_past, c["n_head"],
                               c["n_head_kv"], c["d"], c["eps"], m["cos"], m["sin"])
            np.testing.assert_allclose(got[b], xb, atol=STEP_ATOL, rtol=STEP_RTOL)
        n_past += n
    st.close()


def greedy_decode(torch, ops, m, B, prompt, chunks, steps, penalty=1.1, window=64):
    """Prompt in chunks, then `steps` greedy tokens on the device and in the oracle."""
    W = device_model(ops, m)
    st = new_state(ops, m, B)
    caches = qwen.new_caches(m, B)
    n_past = 0
    for n in chunks:
        tok = prompt[:, n_past:n_past + n]
        x, logits = st.forward_q8(W, dev(torch, tok.astype(np.int32)), n_past)
        x_o, l_o = qwen.forward(m, tok, caches, n_past)
        np.testing.assert_allclose(x.cpu().numpy(), x_o, atol=STEP_ATOL, rtol=STEP_RTOL)
        np.testing.assert_allclose(logits.cpu().numpy(), l_o, atol=STEP_ATOL, rtol=STEP_RTOL)
        n_past += n
    recent = torch.zeros(B, steps, dtype=torch.int32, device="cuda:0")
    recent_o = [[] for _ in range(B)]
    for s in range(steps):
        ops.llm_greedy(logits, recent, n_recent=s, window=window, penalty=penalty, out=recent[:, s])
        for b in range(B):
            recent_o[b].append(qwen.greedy(l_o[b], recent_o[b], window=window, penalty=penalty))
        got = recent[:, s].cpu().numpy().tolist()
        assert got == [r[-1] for r in recent_o], f"step {s}: {got} vs {[r[-1] for r in recent_o]}"
        nxt = recent[:, s:s + 1].contiguous()
        x, logits = st.forward_q8(W, nxt, n_past)
        x_o, l_o = qwen.forward(m, np.array([[r[-1]] for r in recent_o]), caches, n_past)
        np.testing.assert_allclose(logits.cpu().numpy(), l_o, atol=STEP_ATOL, rtol=STEP_RTOL)
        n_past += 1
    st.close()
    return recent.cpu().numpy()


def test_forward_greedy_decode(env):
    """Prompt of 12 tokens in chunks of 8 and 4, then 5 greedy tokens fed back on the device:
    identical tokens, logits within tolerance at every step."""
    torch, ops = env
    m = qwen.make_model(11, n_layer=2, n_vocab=1000, n_head=4, n_head_kv=2, d=64, n_ff=512, n_ctx=64)
    prompt = np.random.default_rng(12).integers(0, 1000, (2, 12))
    greedy_decode(torch, ops, m, 2, prompt, [8, 4], 5)


def test_forward_untied_no_bias_d128(env):
    torch, ops = env
    m = qwen.make_model(13, n_layer=2, n_vocab=2000, n_head=6, n_head_kv=2, d=128, n_ff=1024, n_ctx=32,
                        bias=False, tied=False)
    prompt = np.random.default_rng(14).integers(0, 2000, (3, 5))
    greedy_decode(torch, ops, m, 3, prompt, [5], 3)


def test_chained_launches_in_a_graph(env):
    """The chained (early-starting) launches captured in a CUDA graph and replayed give the
    eager results bit for bit: norm -> q/k/v + RoPE -> attention -> wo + residual -> norm
    -> gate/up -> w_down + residual, i.e. one layer, twice."""
    torch, ops = env
    m = qwen.make_model(15, n_layer=2, n_vocab=100, n_head=4, n_head_kv=2, d=64, n_ff=512, n_ctx=16)
    W = device_model(ops, m)
    B = 4
    rng = np.random.default_rng(16)
    x0 = dev(torch, (rng.standard_normal((B, 1, 256), dtype=np.float32) * 0.5))
    xp = dev(torch, (rng.standard_normal((B, 3, 256), dtype=np.float32) * 0.5))

    def run(st, x, scratch):
        for layer in range(2):
            st.layer_q8(layer, W, x, 3, scratch)

    def prompt(st):
        # positions 0..2 of both states hold the same K/V before the step at n_past = 3
        xs = xp.clone()
        for layer in range(2):
            st.layer_q8(layer, W, xs, 0)

    st_e = new_state(ops, m, B)
    prompt(st_e)
    x_e = x0.clone()
    scratch = st_e.scratch(1, W.n_ff)
    run(st_e, x_e, scratch)
    torch.cuda.synchronize()

    st_g = new_state(ops, m, B)
    prompt(st_g)
    x_g = x0.clone()
    scratch_g = st_g.scratch(1, W.n_ff)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run(st_g, x_g, scratch_g)  # warm-up outside the capture (workspaces sized)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    x_g.copy_(x0)
    with torch.cuda.graph(g):
        run(st_g, x_g, scratch_g)
    for _ in range(3):
        x_g.copy_(x0)
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(x_g, x_e)
    del g
    st_e.close()
    st_g.close()
