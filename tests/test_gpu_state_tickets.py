"""Decode attention through a library state with no per-call ticket clearing.

The split decode kernels (csrc/attn_decode_tma.cu, csrc/attn_decode_tc.cu) merge the pieces
of a segment in the CTA that takes the last ticket, which puts the ticket back to zero. A
state (zwg_llm_state, zwg_dec_state) keeps its tickets in a buffer of its own, cleared when
the state is made and again only after a reported device error, so its calls launch the
kernel alone. These checks run one sequence (16 pieces per segment) through the state's
decode entry point (zwg_llm_attn_decode, the reference's call src/llm.zig:191-202 with n = 1)
many times in a row, eagerly and replayed from a CUDA graph, in both math modes, and once
more after a reported device error, each result against the CPU oracle
(oracle/attention.py, src/ops.zig:562-590)."""
import numpy as np
import pytest

from oracle import attention as A
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu

TOL = {"f32": (1e-4, 0.0), "tf32": (2e-3, 1e-3)}


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import _lib, ops
    yield torch, _lib, ops
    ops.set_math("f32")


def make_state(torch, ops, seed, H=12, Hkv=2, d=128, n_ctx=1024):
    st = ops.LlmState(1, 1, H, Hkv, d, n_ctx)
    kt, v = st.cache_views(0)
    g = torch.Generator(device="cuda:0")
    g.manual_seed(seed)
    kt.copy_(torch.randn(kt.shape, generator=g, device="cuda:0"))
    v.copy_(torch.randn(v.shape, generator=g, device="cuda:0"))
    return st, kt, v


def want_for(st, kt, v, q, n_kv):
    H, Hkv, d, n_ctx = st.n_head, st.n_head_kv, st.d, st.n_ctx
    sh = A.AttnShape(1, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
    return A.attention_ex(q.cpu().numpy().reshape(-1), kt.cpu().numpy().reshape(-1),
                          v.cpu().numpy().reshape(-1), sh)


@pytest.mark.parametrize("math", ["f32", "tf32"])
def test_state_decode_repeated_and_graph(env, math):
    torch, _lib, ops = env
    ops.set_math(math)
    atol, rtol = TOL[math]
    st, kt, v = make_state(torch, ops, seed=11)
    H, d = st.n_head, st.d
    q = torch.randn(1, 1, H * d, device="cuda:0")
    # eager: growing key counts (different piece splits) and the same count twice
    for n_past in (1000, 700, 64, 999, 999):
        out = torch.full_like(q, float("nan"))
        st.attn(0, q, n_past, out=out)
        np.testing.assert_allclose(out.cpu().numpy().reshape(-1), want_for(st, kt, v, q, n_past + 1),
                                   atol=atol, rtol=rtol)
    # a graph of three decode calls, replayed three times with new queries
    out = torch.empty(3, 1, 1, H * d, device="cuda:0")
    qs = torch.empty(3, 1, 1, H * d, device="cuda:0")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for i in range(3):
            st.attn(0, qs[i], 900, out=out[i])
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(3):
            st.attn(0, qs[i], 900, out=out[i])
    for rep in range(3):
        qs.copy_(torch.randn(qs.shape, device="cuda:0"))
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for i in range(3):
            np.testing.assert_allclose(out[i].cpu().numpy().reshape(-1), want_for(st, kt, v, qs[i], 901),
                                       atol=atol, rtol=rtol)
    del graph
    st.close()


def test_state_decode_after_reported_error(env):
    """A reported device error (the bounded-wait self-test) makes the next state call clear
    its tickets first; the results stay exact."""
    torch, _lib, ops = env
    ops.set_math("f32")
    st, kt, v = make_state(torch, ops, seed=12)
    q = torch.randn(1, 1, st.n_head * st.d, device="cuda:0")
    out = torch.empty_like(q)
    st.attn(0, q, 800, out=out)
    lib = _lib.load()
    assert lib.zwg_selftest_timeout() == _lib.ZWG_TIMEOUT
    for _ in range(2):
        out.fill_(float("nan"))
        st.attn(0, q, 800, out=out)
        np.testing.assert_allclose(out.cpu().numpy().reshape(-1), want_for(st, kt, v, q, 801), atol=1e-4, rtol=0)
    st.close()


def test_decoder_state_many_segments(env):
    """32 windows x 8 heads = 256 segments, more than the SMs (whole segments per CTA, no
    ticket): cross-attention over 1500 keys and self-attention over a growing cache through a
    decoder state, each call against the oracle (src/decoder.zig:179-191), three cross calls
    in a row."""
    torch, _lib, ops = env
    ops.set_math("f32")
    B, ns, H, n_text, n_audio = 32, 512, 8, 64, 1500
    st = ops.DecoderState(1, B, ns, H, n_text, n_audio)
    g = torch.Generator(device="cuda:0")
    g.manual_seed(21)
    ck = torch.randn(B, n_audio, ns, generator=g, device="cuda:0")
    cv = torch.randn(B, n_audio, ns, generator=g, device="cuda:0")
    for w in range(B):
        st.set_cross(0, w, ck[w], cv[w])
    ckn, cvn = ck.cpu().numpy(), cv.cpu().numpy()
    for _ in range(3):
        q = torch.randn(B, 1, ns, generator=g, device="cuda:0")
        out = st.cross_attn(0, q).cpu().numpy()
        qn = q.cpu().numpy()
        for b in (0, 13, 31):
            want = A.attention(qn[b].reshape(-1), ckn[b].reshape(-1), cvn[b].reshape(-1), 1, n_audio, ns, H, False)
            np.testing.assert_allclose(out[b].reshape(-1), want, atol=1e-4, rtol=0)
    keys = np.zeros((B, n_text, ns), np.float32)
    vals = np.zeros((B, n_text, ns), np.float32)
    for n_past in range(0, 40, 13):
        q = torch.randn(B, 1, ns, generator=g, device="cuda:0")
        kn = torch.randn(B, 1, ns, generator=g, device="cuda:0")
        vn = torch.randn(B, 1, ns, generator=g, device="cuda:0")
        keys[:, n_past], vals[:, n_past] = kn.cpu().numpy()[:, 0], vn.cpu().numpy()[:, 0]
        out = st.self_attn(0, q, kn, vn, n_past).cpu().numpy()
        qn = q.cpu().numpy()
        for b in (0, 31):
            want = A.attention(qn[b].reshape(-1), keys[b, :n_past + 1].reshape(-1), vals[b, :n_past + 1].reshape(-1),
                               1, n_past + 1, ns, H, True)
            np.testing.assert_allclose(out[b].reshape(-1), want, atol=1e-4, rtol=0)
    st.close()
