"""The library-owned device state of include/zwgpu.h (zwg_dec_state, zwg_llm_state) against
the oracle: a Qwen2 prompt fed in chunks then decoded token by token through
zwg_llm_append_rope + zwg_llm_attn_prefill / _decode (src/llm.zig:168-202), and Whisper
decoder steps through zwg_cross_kv_set + zwg_dec_step_attn (src/decoder.zig:150-191).
The oracle keeps its own caches (oracle/qwen.py, oracle/attention.py) and sees the same
inputs. f32 math is held to abs 1e-4 (the reference's unit-test tolerance,
src/ops.zig:700); the tf32 tensor-core prefill to max-abs 2e-3 with rel 1e-3."""
import numpy as np
import pytest

from oracle import attention as A
from oracle import qwen
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu

F32_ATOL = 1e-4


@pytest.fixture(scope="module")
def env():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    import torch

    from zwhisper_b200 import ops
    ops.set_math("f32")
    return torch, ops


def run_llm(torch, ops, B, L, H, Hkv, d, n_ctx, chunks, seed, atol, rtol=0.0):
    """Feed `chunks` (token counts; 1 = a decode step) through every layer of an LlmState and
    the oracle, comparing rotated q and the attention output of each call."""
    rng = np.random.default_rng(seed)
    dev = torch.device("cuda:0")
    st = ops.LlmState(L, B, H, Hkv, d, n_ctx, rope_base=1e6)
    cos, sin = qwen.rope_tables(n_ctx, d, 1e6)
    kt_o = np.zeros((L, B, Hkv * d * n_ctx), np.float32)
    v_o = np.zeros((L, B, n_ctx * Hkv * d), np.float32)
    n_past = 0
    for n in chunks:
        for layer in range(L):
            q = rng.standard_normal((B, n, H * d), dtype=np.float32)
            k = rng.standard_normal((B, n, Hkv * d), dtype=np.float32)
            v = rng.standard_normal((B, n, Hkv * d), dtype=np.float32)
            tq, tk, tv = (torch.from_numpy(x.copy()).to(dev) for x in (q, k, v))
            st.append_rope(layer, tq, tk, tv, n_past)
            out = st.attn(layer, tq, n_past)
            got_q, got = tq.cpu().numpy(), out.cpu().numpy()
            sho = qwen.attention_call(n, n_past + n, H, Hkv, d, n_ctx)
            for b in range(B):
                qr, _, _ = qwen.rope_and_append(q[b], k[b], v[b], kt_o[layer, b], v_o[layer, b], cos, sin, n_past,
                                                H, Hkv, d)
                np.testing.assert_allclose(got_q[b], qr, atol=1e-5, rtol=0)
                want = A.attention_ex(qr.reshape(-1), kt_o[layer, b], v_o[layer, b], sho)
                np.testing.assert_allclose(got[b].reshape(-1), want, atol=atol, rtol=rtol)
        n_past += n
    ptrs = st.cache_ptrs(0)
    assert all(p for p in ptrs)
    st.close()


def test_llm_state_prompt_then_decode(env):
    torch, ops = env
    # a 300-token prompt in chunks of 128 (the reference's batch is 256) then 3 decode steps
    run_llm(torch, ops, B=2, L=2, H=14, Hkv=2, d=64, n_ctx=512, chunks=[128, 128, 44, 1, 1, 1], seed=1,
            atol=F32_ATOL)


def test_llm_state_d128_decode(env):
    torch, ops = env
    run_llm(torch, ops, B=3, L=1, H=12, Hkv=2, d=128, n_ctx=256, chunks=[37, 1, 1], seed=2, atol=F32_ATOL)


def test_llm_state_tf32_prefill(env):
    """With the math mode at tf32 the prefill chunks run on the tensor-core kernel."""
    torch, ops = env
    ops.set_math("tf32")
    try:
        run_llm(torch, ops, B=2, L=1, H=12, Hkv=2, d=128, n_ctx=512, chunks=[256, 200, 1], seed=3,
                atol=2e-3, rtol=1e-3)
    finally:
        ops.set_math("f32")


def test_llm_state_context_full_is_an_error(env):
    torch, ops = env
    from zwhisper_b200 import _lib
    st = ops.LlmState(1, 1, 2, 1, 64, 64)
    q = torch.zeros(1, 65, 128, device="cuda:0")
    k = torch.zeros(1, 65, 64, device="cuda:0")
    with pytest.raises(_lib.ZwgError, match="context full"):
        st.append_rope(0, q, k, k.clone(), 0)
    st.close()


def test_decoder_state_steps(env):
    """Three windows, two layers: a 3-token prompt then two single-token steps, self then
    cross attention per layer, as the decoder runs them (src/decoder.zig:166-191)."""
    torch, ops = env
    rng = np.random.default_rng(4)
    dev = torch.device("cuda:0")
    B, L, ns, H, n_text, n_audio = 3, 2, 512, 8, 448, 1500
    st = ops.DecoderState(L, B, ns, H, n_text, n_audio)
    ck = rng.standard_normal((L, B, n_audio, ns), dtype=np.float32)
    cv = rng.standard_normal((L, B, n_audio, ns), dtype=np.float32)
    for layer in range(L):
        for w in range(B):
            # device tensors for layer 0, pinned host tensors for layer 1 (both accepted)
            tk = torch.from_numpy(ck[layer, w].copy())
            tv = torch.from_numpy(cv[layer, w].copy())
            if layer == 0:
                tk, tv = tk.to(dev), tv.to(dev)
            else:
                tk, tv = tk.pin_memory(), tv.pin_memory()
            st.set_cross(layer, w, tk, tv)
    torch.cuda.synchronize()
    sk = np.zeros((L, B, n_text, ns), np.float32)
    sv = np.zeros((L, B, n_text, ns), np.float32)
    n_past = 0
    for n in (3, 1, 1):
        for layer in range(L):
            q = rng.standard_normal((B, n, ns), dtype=np.float32)
            k = rng.standard_normal((B, n, ns), dtype=np.float32)
            v = rng.standard_normal((B, n, ns), dtype=np.float32)
            qc = rng.standard_normal((B, n, ns), dtype=np.float32)
            tq, tk, tv, tqc = (torch.from_numpy(x).to(dev) for x in (q, k, v, qc))
            got_s = st.self_attn(layer, tq, tk, tv, n_past).cpu().numpy()
            got_c = st.cross_attn(layer, tqc).cpu().numpy()
            sk[layer, :, n_past:n_past + n] = k
            sv[layer, :, n_past:n_past + n] = v
            n_kv = n_past + n
            for w in range(B):
                want_s = A.attention(q[w].reshape(-1), sk[layer, w, :n_kv].reshape(-1), sv[layer, w, :n_kv].reshape(-1),
                                     n, n_kv, ns, H, True)
                want_c = A.attention(qc[w].reshape(-1), ck[layer, w].reshape(-1), cv[layer, w].reshape(-1),
                                     n, n_audio, ns, H, False)
                np.testing.assert_allclose(got_s[w].reshape(-1), want_s, atol=F32_ATOL, rtol=0)
                np.testing.assert_allclose(got_c[w].reshape(-1), want_c, atol=F32_ATOL, rtol=0)
        n_past += n
    assert all(p for p in st.cache_ptrs(1))
    st.close()
