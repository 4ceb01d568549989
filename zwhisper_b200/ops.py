"""Host-side mirror of the reference's attention operator interface (src/ops.zig:464-605),
running on the B200 through libzwgpu.

Same names, argument meaning and error behaviour as the reference:
  - `AttnShape` mirrors ops.AttnShape (src/ops.zig:477-492);
  - `attention_ex(q, k, v, sh, scratch, out)` mirrors ops.attentionEx (src/ops.zig:562) on
    host float32 arrays, synchronously (the pool argument has no counterpart);
  - `attention(...)` mirrors ops.attention (src/ops.zig:593);
  - `attention_scratch_ex / _kt / attention_scratch` mirror the sizers
    (src/ops.zig:545-560) and return the device workspace in floats.
Shape violations the reference asserts on (src/ops.zig:564-568) raise ValueError here.

Device entry points (torch tensors on a CUDA device, stream ordered on the current torch
stream): `attention_dev`, `enc_attn_bf16`, `rope_kt_append`, `f32_to_bf16`; the library-owned
states `DecoderState` and `LlmState`; the Q8 projections `quantize_q8`, `linear_q8`,
`linear_q8_add`, `linear_q8_silu_mul`; and the rest of the Qwen2 decode step (src/llm.zig:
168-216, 268-321): `rms_norm`, `embed_q8`, `llm_greedy`, `LlmWeightsQ8` with
`LlmState.qkv_q8 / layer_q8 / forward_q8`; and the Whisper decoder step (src/decoder.zig:
151-206): `layer_norm`, `linear_q8_gelu`, `DecoderWeightsQ8` with
`DecoderState.set_audio_q8 / forward_q8`.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _lib

Q_BLOCK = 64  # src/ops.zig:473, kept for callers that size buffers by it


@dataclass
class AttnShape:
    """ops.AttnShape (src/ops.zig:477-492). Strides in floats. kt_stride=None: keys are rows."""

    n_q: int
    n_kv: int
    n_head: int
    n_head_kv: int
    d: int
    q_stride: int
    kv_stride: int
    out_stride: int
    causal: bool
    kt_stride: Optional[int] = None

    def to_c(self) -> _lib.AttnShapeC:
        return _lib.AttnShapeC(self.n_q, self.n_kv, self.n_head, self.n_head_kv, self.d, self.q_stride,
                               self.kv_stride, self.out_stride, 1 if self.causal else 0, self.kt_stride or 0)

    def extents(self):
        """Elements of q, k, v, out that the call reads or writes."""
        def span(rows, stride, width):
            return (rows - 1) * stride + width if rows else 0
        q = span(self.n_q, self.q_stride, self.n_head * self.d)
        if self.kt_stride:
            k = self.n_head_kv * self.d * self.kt_stride
        else:
            k = span(self.n_kv, self.kv_stride, self.n_head_kv * self.d)
        v = span(self.n_kv, self.kv_stride, self.n_head_kv * self.d)
        out = span(self.n_q, self.out_stride, self.n_head * self.d)
        return q, k, v, out


def mha_shape(n_q: int, n_kv: int, n_state: int, n_head: int, causal: bool) -> AttnShape:
    """The shape ops.attention builds (src/ops.zig:593-605)."""
    if n_head <= 0 or n_state % n_head:
        raise ValueError(f"n_state {n_state} is not a multiple of n_head {n_head}")
    return AttnShape(n_q, n_kv, n_head, n_head, n_state // n_head, n_state, n_state, n_state, causal)


def _validate(sh: AttnShape) -> None:
    if sh.n_head_kv <= 0 or sh.n_head % sh.n_head_kv:
        raise ValueError("n_head must be a positive multiple of n_head_kv")
    if sh.causal and sh.n_kv < sh.n_q:
        raise ValueError("causal attention needs n_kv >= n_q")


def _host_f32(a, n: int, name: str) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    if a.size < n:
        raise ValueError(f"{name} holds {a.size} floats, the shape needs {n}")
    return a


def attention_ex(q, k, v, sh: AttnShape, scratch=None, out=None, device: int = 0) -> np.ndarray:
    """ops.attentionEx (src/ops.zig:562) on the GPU: host float32 in, host float32 out."""
    _validate(sh)
    nq, nk, nv, no = sh.extents()
    q = _host_f32(q, nq, "q")
    k = _host_f32(k, nk, "k")
    v = _host_f32(v, nv, "v")
    if out is None:
        out = np.zeros(max(no, 1), np.float32)
    elif not (isinstance(out, np.ndarray) and out.dtype == np.float32 and out.flags.c_contiguous):
        raise ValueError("out must be a contiguous float32 numpy array")
    if out.size < no:
        raise ValueError(f"out holds {out.size} floats, the shape needs {no}")
    _lib.ensure_init(device)
    lib = _lib.load()
    c = sh.to_c()
    _lib.check(lib.zwg_attention(ctypes.byref(c), q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data))
    return out


def attention(q, k, v, n_q: int, n_kv: int, n_state: int, n_head: int, causal: bool, scratch=None, out=None,
              device: int = 0) -> np.ndarray:
    """ops.attention (src/ops.zig:593)."""
    return attention_ex(q, k, v, mha_shape(n_q, n_kv, n_state, n_head, causal), scratch, out, device)


def attention_batch_host(q, k, v, sh: AttnShape, n_batch: int, out=None, device: int = 0) -> np.ndarray:
    """attentionEx over n_batch independent host items laid out back to back, with copies
    pipelined against compute (zwg_attention_batch_host)."""
    _validate(sh)
    nq, nk, nv, no = sh.extents()
    q = _host_f32(q, nq * n_batch, "q")
    k = _host_f32(k, nk * n_batch, "k")
    v = _host_f32(v, nv * n_batch, "v")
    if out is None:
        out = np.zeros(max(no * n_batch, 1), np.float32)
    _lib.ensure_init(device)
    lib = _lib.load()
    c = sh.to_c()
    b = _lib.BatchC(n_batch, nq, nk, nv, no)
    _lib.check(lib.zwg_attention_batch_host(ctypes.byref(c), ctypes.byref(b), q.ctypes.data, k.ctypes.data,
                                            v.ctypes.data, out.ctypes.data))
    return out


def set_math(mode: str, device: int = 0) -> None:
    """Math mode of the calling thread's context (zwg_set_math): "f32" (default, the
    reference's arithmetic), "bf16" (encoder-shaped host calls on the bf16 tcgen05 kernel),
    "tf32" (prefill calls over a transposed key cache on the tf32 tcgen05 kernel), or
    "bf16+tf32" for both."""
    _lib.ensure_init(device)
    code = 0
    for part in mode.split("+"):
        code |= {"f32": _lib.ZWG_MATH_F32, "bf16": _lib.ZWG_MATH_BF16, "tf32": _lib.ZWG_MATH_TF32}[part]
    _lib.check(_lib.load().zwg_set_math(code))


def q8_tensor_cores(enable=None) -> int:
    """Where Q8 products of 16 or more rows with k a multiple of 64 run (zwg_q8_tensor_cores,
    process-wide): 1 / True (default) on the tcgen05 kernel except small products at up to
    64 rows (k <= 1024, at most 1.25 M weights), 2 / "always" on the tcgen05 kernel for every
    such product, 0 / False on the CUDA-core kernel. With an argument, sets it and returns
    the previous setting; without, returns the current one."""
    if enable is None:
        code = -1
    elif enable == "always":
        code = 2
    else:
        code = int(enable)
    return int(_lib.load().zwg_q8_tensor_cores(code))


# ---- scratch sizers (src/ops.zig:545-560): device workspace in floats ----------------------

def attention_workspace_bytes(sh: AttnShape, n_batch: int = 1) -> int:
    lib = _lib.load()
    c = sh.to_c()
    b = _lib.BatchC(n_batch, 0, 0, 0, 0)
    return int(lib.zwg_attention_workspace(ctypes.byref(c), ctypes.byref(b)))


def attention_scratch_ex(n_q, n_kv, n_head, n_head_kv, d) -> int:
    sh = AttnShape(n_q, n_kv, n_head, n_head_kv, d, n_head * d, n_head_kv * d, n_head * d, False)
    return attention_workspace_bytes(sh) // 4


def attention_scratch_kt(n_q, kt_stride, n_head, n_head_kv=None, d=64) -> int:
    n_head_kv = n_head_kv or n_head
    sh = AttnShape(n_q, kt_stride, n_head, n_head_kv, d, n_head * d, n_head_kv * d, n_head * d, True, kt_stride)
    return attention_workspace_bytes(sh) // 4


def attention_scratch(n_q, n_kv, n_head, n_state) -> int:
    return attention_scratch_ex(n_q, n_kv, n_head, n_head, n_state // n_head)


# ---- device (torch) entry points -----------------------------------------------------------

def _torch():
    import torch
    return torch


def _dev_ptr(t, dtype, name):
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _stream_of(t):
    torch = _torch()
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def attention_dev(q, k, v, sh: AttnShape, out, n_batch: int = 1, batch_strides=None, workspace=None):
    """attentionEx on device f32 tensors over n_batch items (zwg_attention_dev).

    batch_strides: (q, k, v, out) element strides between items; default = each tensor's
    numel / n_batch. workspace: a CUDA uint8 tensor of at least attention_workspace_bytes."""
    torch = _torch()
    _validate(sh)
    _lib.ensure_init(q.device.index or 0)
    if batch_strides is None:
        batch_strides = tuple(t.numel() // n_batch for t in (q, k, v, out))
    c = sh.to_c()
    b = _lib.BatchC(n_batch, *batch_strides)
    need = attention_workspace_bytes(sh, n_batch)
    if workspace is None and need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if workspace is not None else 0
    ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
    lib = _lib.load()
    _lib.check(lib.zwg_attention_dev(ctypes.byref(c), ctypes.byref(b), _dev_ptr(q, torch.float32, "q"),
                                     _dev_ptr(k, torch.float32, "k"), _dev_ptr(v, torch.float32, "v"),
                                     _dev_ptr(out, torch.float32, "out"), ws_ptr, ws_len, _stream_of(q)))
    return out


def enc_attn_bf16(q, k, v, n_head: int, out=None):
    """Encoder self-attention on tcgen05 tensor cores: bf16 q, k, v [B][n_ctx][n_head*64],
    f32 out of the same shape (zwg_enc_attn_bf16)."""
    torch = _torch()
    if q.dim() != 3 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must share one [B][n_ctx][n_state] shape")
    B, n_ctx, ns = q.shape
    if ns != n_head * 64:
        raise ValueError("head dim must be 64")
    if out is None:
        out = torch.empty(B, n_ctx, ns, dtype=torch.float32, device=q.device)
    _lib.ensure_init(q.device.index or 0)
    lib = _lib.load()
    _lib.check(lib.zwg_enc_attn_bf16(B, n_ctx, n_head, _dev_ptr(q, torch.bfloat16, "q"),
                                     _dev_ptr(k, torch.bfloat16, "k"), _dev_ptr(v, torch.bfloat16, "v"),
                                     _dev_ptr(out, torch.float32, "out"), _stream_of(q)))
    return out


def f32_to_bf16(x, out=None):
    torch = _torch()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.ensure_init(x.device.index or 0)
    _lib.check(_lib.load().zwg_f32_to_bf16(_dev_ptr(x, torch.float32, "x"), _dev_ptr(out, torch.bfloat16, "out"),
                                           x.numel(), _stream_of(x)))
    return out


def rope_tables(n_ctx: int, d: int, base: float):
    """cos/sin [n_ctx][d/2] f32: inverse frequencies base^(-2i/d) and angles in f64, cast to
    f32 (src/llm.zig:128-137)."""
    half = d // 2
    i = np.arange(half, dtype=np.float64)
    inv = 1.0 / np.power(np.float64(base), 2.0 * i / np.float64(d))
    ang = np.arange(n_ctx, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope_kt_append(q, k, v, cache_kt, cache_v, cos_t, sin_t, n_past: int, n_head: int, n_head_kv: int, d: int,
                   n_ctx: int, n_batch: int = 1):
    """Qwen2 RoPE on q (in place) and k, then append k into the transposed cache and v into
    the value cache at positions n_past.. (src/llm.zig:182-190, 221-238)."""
    torch = _torch()
    n = q.numel() // n_batch // (n_head * d)
    _lib.ensure_init(q.device.index or 0)
    _lib.check(_lib.load().zwg_rope_kt_append(
        n_batch, n, n_past, n_head, n_head_kv, d, n_ctx, _dev_ptr(q, torch.float32, "q"),
        _dev_ptr(k, torch.float32, "k"), _dev_ptr(v, torch.float32, "v"), _dev_ptr(cache_kt, torch.float32, "cache_kt"),
        _dev_ptr(cache_v, torch.float32, "cache_v"), _dev_ptr(cos_t, torch.float32, "cos"),
        _dev_ptr(sin_t, torch.float32, "sin"), q.numel() // n_batch, k.numel() // n_batch,
        cache_kt.numel() // n_batch, _stream_of(q)))


def sync() -> None:
    _lib.check(_lib.load().zwg_sync())


# ---- library-owned device state (zwg_dec_state / zwg_llm_state) ----------------------------

def _check_rows(t, n_batch: int, n: int, width: int, name: str):
    if t.numel() != n_batch * n * width:
        raise ValueError(f"{name} must hold n_batch * n * {width} floats, got {t.numel()}")


class DecoderState:
    """Whisper decoder attention state on one device (zwg_dec_state): per layer the self
    K/V cache [n_batch][n_text_ctx][n_state] and the cross K/V [n_batch][n_audio_ctx][n_state]
    (src/decoder.zig:39-42, 127-130)."""

    def __init__(self, n_layer: int, n_batch: int, n_state: int, n_head: int, n_text_ctx: int = 448,
                 n_audio_ctx: int = 1500, device: int = 0):
        _lib.ensure_init(device)
        self.device, self.n_layer, self.n_batch = device, n_layer, n_batch
        self.n_state, self.n_head, self.n_text_ctx, self.n_audio_ctx = n_state, n_head, n_text_ctx, n_audio_ctx
        h = ctypes.c_void_p()
        _lib.check(_lib.load().zwg_dec_state_create(n_layer, n_batch, n_state, n_head, n_text_ctx, n_audio_ctx,
                                                    ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            _lib.check(_lib.load().zwg_dec_state_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def cache_ptrs(self, layer: int):
        """Device addresses (self_k, self_v, cross_k, cross_v) of one layer."""
        p = [ctypes.c_void_p() for _ in range(4)]
        _lib.check(_lib.load().zwg_dec_state_cache(self._h, layer, *(ctypes.byref(x) for x in p)))
        return tuple(x.value for x in p)

    def cache_views(self, layer: int):
        """Torch views (no copy) of one layer's buffers: self K, self V [n_batch][n_text_ctx]
        [n_state] and cross K, cross V [n_batch][n_audio_ctx][n_state]. Valid until close()."""
        torch = _torch()
        ptrs = self.cache_ptrs(layer)
        dev = torch.device("cuda", self.device)
        shapes = [(self.n_batch, self.n_text_ctx, self.n_state)] * 2 + [(self.n_batch, self.n_audio_ctx, self.n_state)] * 2
        return tuple(torch.as_tensor(_DeviceArray(p, shp), device=dev) for p, shp in zip(ptrs, shapes))

    def set_cross(self, layer: int, window: int, k, v) -> None:
        """setAudio for one window and layer (src/decoder.zig:150-156): k, v [n_audio_ctx][n_state]."""
        torch = _torch()
        for t, name in ((k, "k"), (v, "v")):
            if t.numel() != self.n_audio_ctx * self.n_state or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous f32 [n_audio_ctx][n_state]")
        stream = _stream_of(k) if k.is_cuda else None
        _lib.check(_lib.load().zwg_cross_kv_set(self._h, layer, window, k.data_ptr(), v.data_ptr(), stream))

    def self_attn(self, layer: int, q, k_new, v_new, n_past: int, out=None):
        """Append k_new/v_new at n_past.. and attend causally (src/decoder.zig:179-184);
        q, k_new, v_new, out [n_batch][n][n_state] CUDA f32."""
        torch = _torch()
        n = q.numel() // (self.n_batch * self.n_state)
        for t, name in ((q, "q"), (k_new, "k_new"), (v_new, "v_new")):
            _check_rows(t, self.n_batch, n, self.n_state, name)
        out = torch.empty_like(q) if out is None else out
        _lib.check(_lib.load().zwg_dec_step_attn(
            self._h, layer, _lib.ZWG_DEC_SELF, _dev_ptr(q, torch.float32, "q"), _dev_ptr(k_new, torch.float32, "k_new"),
            _dev_ptr(v_new, torch.float32, "v_new"), n_past, n, _dev_ptr(out, torch.float32, "out"), _stream_of(q)))
        return out

    def cross_attn(self, layer: int, q, out=None):
        """Attention over each window's cross K/V (src/decoder.zig:188-191)."""
        torch = _torch()
        n = q.numel() // (self.n_batch * self.n_state)
        _check_rows(q, self.n_batch, n, self.n_state, "q")
        out = torch.empty_like(q) if out is None else out
        _lib.check(_lib.load().zwg_dec_step_attn(
            self._h, layer, _lib.ZWG_DEC_CROSS, _dev_ptr(q, torch.float32, "q"), None, None, 0, n,
            _dev_ptr(out, torch.float32, "out"), _stream_of(q)))
        return out


    def set_audio_q8(self, weights: "DecoderWeightsQ8", window: int, enc) -> None:
        """setAudio (src/decoder.zig:151-159) on the device: enc [n_audio_ctx][n_state] (CUDA
        f32) -> every layer's cross K/V of `window`."""
        torch = _torch()
        if enc.numel() != self.n_audio_ctx * self.n_state:
            raise ValueError("enc must hold n_audio_ctx * n_state floats")
        _lib.check(_lib.load().zwg_dec_set_audio_q8(self._h, ctypes.byref(weights.c_struct()), window,
                                                    _dev_ptr(enc, torch.float32, "enc"), _stream_of(enc)))

    def scratch(self, n: int, scratch=None):
        """A CUDA uint8 buffer of at least zwg_dec_scratch_bytes for chunks of n tokens."""
        torch = _torch()
        need = _lib.load().zwg_dec_scratch_bytes(self._h, n)
        if scratch is None or scratch.numel() < need:
            scratch = torch.empty(max(need, 256), dtype=torch.uint8, device=torch.device("cuda", self.device))
        return scratch

    def forward_q8(self, weights: "DecoderWeightsQ8", tokens, n_past: int, x=None, logits=None, scratch=None):
        """Decoder.forward (src/decoder.zig:166-206) for every window: tokens CUDA int32
        [n_batch][n] at positions n_past..; returns (x [n_batch][n][n_state], logits
        [n_batch][n_vocab] of each window's last token)."""
        torch = _torch()
        if tokens.dtype != torch.int32 or not tokens.is_contiguous() or tokens.numel() % self.n_batch:
            raise ValueError("tokens must be a contiguous int32 [n_batch][n] tensor")
        n = tokens.numel() // self.n_batch
        dev = tokens.device
        if x is None:
            x = torch.empty(self.n_batch, n, self.n_state, dtype=torch.float32, device=dev)
        if logits is None:
            logits = torch.empty(self.n_batch, weights.n_vocab, dtype=torch.float32, device=dev)
        scratch = self.scratch(n, scratch)
        _lib.check(_lib.load().zwg_dec_forward_q8(self._h, ctypes.byref(weights.c_struct()), tokens.data_ptr(),
                                                  n_past, n, _dev_ptr(x, torch.float32, "x"),
                                                  _dev_ptr(logits, torch.float32, "logits"), scratch.data_ptr(),
                                                  scratch.numel(), _stream_of(tokens)))
        return x, logits

class _DeviceArray:
    """A float32 device buffer described by __cuda_array_interface__ (for zero-copy views)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class LlmState:
    """Qwen2 attention state on one device (zwg_llm_state): per layer cache_kt
    [n_batch][n_head_kv][d][n_ctx] and cache_v [n_batch][n_ctx][n_head_kv*d], RoPE tables in
    f64 (src/llm.zig:27-28, 124-137)."""

    def __init__(self, n_layer: int, n_batch: int, n_head: int, n_head_kv: int, d: int, n_ctx: int,
                 rope_base: float = 1e6, device: int = 0):
        _lib.ensure_init(device)
        self.device, self.n_layer, self.n_batch = device, n_layer, n_batch
        self.n_head, self.n_head_kv, self.d, self.n_ctx = n_head, n_head_kv, d, n_ctx
        h = ctypes.c_void_p()
        _lib.check(_lib.load().zwg_llm_state_create(n_layer, n_batch, n_head, n_head_kv, d, n_ctx, float(rope_base),
                                                    ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            _lib.check(_lib.load().zwg_llm_state_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def cache_ptrs(self, layer: int):
        """Device addresses (cache_kt, cache_v) of one layer."""
        kt, v = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(_lib.load().zwg_llm_state_cache(self._h, layer, ctypes.byref(kt), ctypes.byref(v)))
        return kt.value, v.value

    def cache_views(self, layer: int):
        """Torch views (no copy) of one layer's caches: cache_kt [n_batch][n_head_kv][d][n_ctx]
        and cache_v [n_batch][n_ctx][n_head_kv*d]. Valid until close()."""
        torch = _torch()
        kt, v = self.cache_ptrs(layer)
        dev = torch.device("cuda", self.device)
        shapes = ((self.n_batch, self.n_head_kv, self.d, self.n_ctx),
                  (self.n_batch, self.n_ctx, self.n_head_kv * self.d))
        return tuple(torch.as_tensor(_DeviceArray(p, shp), device=dev) for p, shp in zip((kt, v), shapes))

    def append_rope(self, layer: int, q, k, v, n_past: int) -> None:
        """RoPE on q (in place) and k, cache append at n_past.. (src/llm.zig:180-190)."""
        torch = _torch()
        n = q.numel() // (self.n_batch * self.n_head * self.d)
        _check_rows(q, self.n_batch, n, self.n_head * self.d, "q")
        _check_rows(k, self.n_batch, n, self.n_head_kv * self.d, "k")
        _check_rows(v, self.n_batch, n, self.n_head_kv * self.d, "v")
        _lib.check(_lib.load().zwg_llm_append_rope(
            self._h, layer, _dev_ptr(q, torch.float32, "q"), _dev_ptr(k, torch.float32, "k"),
            _dev_ptr(v, torch.float32, "v"), n_past, n, _stream_of(q)))

    def attn(self, layer: int, q, n_past: int, out=None):
        """Causal GQA attention over the cache, n_kv = n_past + n (src/llm.zig:191-202);
        n = 1 runs zwg_llm_attn_decode, otherwise zwg_llm_attn_prefill."""
        torch = _torch()
        n = q.numel() // (self.n_batch * self.n_head * self.d)
        _check_rows(q, self.n_batch, n, self.n_head * self.d, "q")
        out = torch.empty_like(q) if out is None else out
        lib = _lib.load()
        if n == 1:
            rc = lib.zwg_llm_attn_decode(self._h, layer, _dev_ptr(q, torch.float32, "q"), n_past,
                                         _dev_ptr(out, torch.float32, "out"), _stream_of(q))
        else:
            rc = lib.zwg_llm_attn_prefill(self._h, layer, _dev_ptr(q, torch.float32, "q"), n_past, n,
                                          _dev_ptr(out, torch.float32, "out"), _stream_of(q))
        _lib.check(rc)
        return out

    def qkv_q8(self, layer: int, x, weights: "LlmWeightsQ8", n_past: int, q_out=None):
        """The q/k/v projections with bias, RoPE and the cache append in one launch
        (src/llm.zig:179-190): x [n_batch][n][n_head*d] normed hidden states; returns the rotated
        q and writes k, v into the layer's caches at n_past.."""
        torch = _torch()
        width = self.n_head * self.d
        n = x.numel() // (self.n_batch * width)
        _check_rows(x, self.n_batch, n, width, "x")
        q_out = torch.empty_like(x) if q_out is None else q_out
        lw = weights.layer_c(layer)
        _lib.check(_lib.load().zwg_llm_qkv_q8(self._h, layer, _dev_ptr(x, torch.float32, "x"), ctypes.byref(lw), n_past,
                                              n, _dev_ptr(q_out, torch.float32, "q_out"), _stream_of(x)))
        return q_out


    def scratch(self, n: int, n_ff: int, scratch=None):
        """A CUDA uint8 buffer of at least zwg_llm_scratch_bytes for chunks of n tokens."""
        torch = _torch()
        need = _lib.load().zwg_llm_scratch_bytes(self._h, n, n_ff)
        if scratch is None or scratch.numel() < need:
            scratch = torch.empty(max(need, 256), dtype=torch.uint8, device=torch.device("cuda", self.device))
        return scratch


    def layer_q8(self, layer: int, weights: "LlmWeightsQ8", x, n_past: int, scratch=None):
        """One layer of Model.forward (src/llm.zig:177-210) on x [n_batch][n][n_embd], in place."""
        torch = _torch()
        n = x.numel() // (self.n_batch * weights.n_embd)
        _check_rows(x, self.n_batch, n, weights.n_embd, "x")
        scratch = self.scratch(n, weights.n_ff, scratch)
        _lib.check(_lib.load().zwg_llm_layer_q8(self._h, layer, ctypes.byref(weights.c_struct()),
                                                _dev_ptr(x, torch.float32, "x"), n_past, n, scratch.data_ptr(),
                                                scratch.numel(), _stream_of(x)))
        return x


    def forward_q8(self, weights: "LlmWeightsQ8", tokens, n_past: int, x=None, logits=None, scratch=None):
        """Model.forward (src/llm.zig:169-216) for every sequence: tokens CUDA int32
        [n_batch][n] at positions n_past..; returns (x [n_batch][n][n_embd], logits
        [n_batch][n_vocab] of each sequence's last token)."""
        torch = _torch()
        if tokens.dtype != torch.int32 or not tokens.is_contiguous() or tokens.numel() % self.n_batch:
            raise ValueError("tokens must be a contiguous int32 [n_batch][n] tensor")
        n = tokens.numel() // self.n_batch
        dev = tokens.device
        if x is None:
            x = torch.empty(self.n_batch, n, weights.n_embd, dtype=torch.float32, device=dev)
        if logits is None:
            logits = torch.empty(self.n_batch, weights.n_vocab, dtype=torch.float32, device=dev)
        scratch = self.scratch(n, weights.n_ff, scratch)
        _lib.check(_lib.load().zwg_llm_forward_q8(self._h, ctypes.byref(weights.c_struct()), tokens.data_ptr(), n_past,
                                                  n, _dev_ptr(x, torch.float32, "x"),
                                                  _dev_ptr(logits, torch.float32, "logits"), scratch.data_ptr(),
                                                  scratch.numel(), _stream_of(tokens)))
        return x, logits


# ---- Q8 weights (zwg_q8_quantize / zwg_linear_q8) ------------------------------------------

def quantize_q8(w):
    """Q8.quantize (src/gemm.zig:208-230) of a CUDA f32 [n][k] tensor: (q int8 [n][k],
    scales f32 [n][k/32]), bit-identical to the reference."""
    torch = _torch()
    n, k = w.shape
    q = torch.empty(n, k, dtype=torch.int8, device=w.device)
    s = torch.empty(n, k // 32, dtype=torch.float32, device=w.device)
    _lib.ensure_init(w.device.index or 0)
    _lib.check(_lib.load().zwg_q8_quantize(_dev_ptr(w, torch.float32, "w"), n, k, q.data_ptr(), s.data_ptr(),
                                           _stream_of(w)))
    return q, s


def linear_q8(x, q, scales, bias=None, out=None):
    """ops.linear with Q8 weights (src/ops.zig:280-306): out[m][n] = x[m][k] . W[n][k]^T + b."""
    torch = _torch()
    m, k = x.shape
    n = q.shape[0]
    if q.shape[1] != k or q.dtype != torch.int8 or not q.is_contiguous():
        raise ValueError("q must be contiguous int8 [n][k]")
    if scales.numel() != n * (k // 32):
        raise ValueError("scales must hold n * k / 32 floats")
    out = torch.empty(m, n, dtype=torch.float32, device=x.device) if out is None else out
    _lib.ensure_init(x.device.index or 0)
    _lib.check(_lib.load().zwg_linear_q8(
        _dev_ptr(x, torch.float32, "x"), m, k, q.data_ptr(), _dev_ptr(scales, torch.float32, "scales"),
        _dev_ptr(bias, torch.float32, "bias") if bias is not None else None, n,
        _dev_ptr(out, torch.float32, "out"), _stream_of(x)))
    return out


# ---- the Qwen2 decode step around the attention (src/llm.zig:168-216, 268-321) -----------

def _q8_pair(w, name):
    """(q int8 [n][k], scales f32 [n][k/32]) on the device, checked."""
    torch = _torch()
    q, s = w
    if q.dtype != torch.int8 or not q.is_cuda or not q.is_contiguous():
        raise ValueError(f"{name}: q must be a contiguous CUDA int8 tensor")
    if s.numel() != q.shape[0] * (q.shape[1] // 32):
        raise ValueError(f"{name}: scales must hold n * k / 32 floats")
    return q, _dev_ptr(s, torch.float32, f"{name} scales")


def rms_norm(x, w, eps: float, out=None):
    """ops.rmsNorm (src/ops.zig:408-425) of the rows of a CUDA f32 [m][n] tensor."""
    torch = _torch()
    n = x.shape[-1]
    m = x.numel() // n
    out = torch.empty_like(x) if out is None else out
    _lib.ensure_init(x.device.index or 0)
    _lib.check(_lib.load().zwg_rms_norm(_dev_ptr(x, torch.float32, "x"), m, n, _dev_ptr(w, torch.float32, "w"),
                                        float(eps), _dev_ptr(out, torch.float32, "out"), _stream_of(x)))
    return out


def linear_q8_add(x, q, scales, out):
    """out += x . W^T (ops.linear then ops.add, src/llm.zig:203-204) with Q8 W; returns out."""
    torch = _torch()
    m, k = x.shape
    q, sp = _q8_pair((q, scales), "w")
    if q.shape[1] != k:
        raise ValueError("q must be [n][k]")
    _lib.ensure_init(x.device.index or 0)
    _lib.check(_lib.load().zwg_linear_q8_add(_dev_ptr(x, torch.float32, "x"), m, k, q.data_ptr(), sp, q.shape[0],
                                             _dev_ptr(out, torch.float32, "out"), _stream_of(x)))
    return out


def linear_q8_silu_mul(x, gate, up, out=None):
    """silu(x . Wg^T) * (x . Wu^T) in one launch (src/llm.zig:206-208, src/ops.zig:435-440);
    gate and up are (q, scales) pairs of the same shape."""
    torch = _torch()
    m, k = x.shape
    gq, gs = _q8_pair(gate, "gate")
    uq, us = _q8_pair(up, "up")
    if gq.shape != uq.shape or gq.shape[1] != k:
        raise ValueError("gate and up must both be [n][k]")
    n = gq.shape[0]
    out = torch.empty(m, n, dtype=torch.float32, device=x.device) if out is None else out
    _lib.ensure_init(x.device.index or 0)
    _lib.check(_lib.load().zwg_linear_q8_silu_mul(_dev_ptr(x, torch.float32, "x"), m, k, gq.data_ptr(), gs,
                                                  uq.data_ptr(), us, n, _dev_ptr(out, torch.float32, "out"),
                                                  _stream_of(x)))
    return out


def embed_q8(tokens, q, scales, out=None):
    """Q8.row (src/gemm.zig:256-263) of each token id (CUDA int32): out [m][k] f32."""
    torch = _torch()
    if tokens.dtype != torch.int32 or not tokens.is_cuda or not tokens.is_contiguous():
        raise ValueError("tokens must be a contiguous CUDA int32 tensor")
    q, sp = _q8_pair((q, scales), "embd")
    m = tokens.numel()
    out = torch.empty(m, q.shape[1], dtype=torch.float32, device=tokens.device) if out is None else out
    _lib.ensure_init(tokens.device.index or 0)
    _lib.check(_lib.load().zwg_embed_q8(tokens.data_ptr(), m, q.data_ptr(), sp, q.shape[0], q.shape[1],
                                        _dev_ptr(out, torch.float32, "out"), _stream_of(tokens)))
    return out


def llm_greedy(logits, recent=None, n_recent: int = 0, window: int = 64, penalty: float = 1.1, out=None):
    """Model.penalize then Model.argmax (src/llm.zig:268-273, 313-321) for each row of
    logits [m][n_vocab] (penalized in place). recent: CUDA int32 [m][>= n_recent], the tokens
    generated so far; out: a CUDA int32 [m] tensor or a column view such as recent[:, i]."""
    torch = _torch()
    m, n_vocab = logits.shape
    if not logits.is_contiguous():
        raise ValueError("logits must be contiguous")
    if out is None:
        out = torch.empty(m, dtype=torch.int32, device=logits.device)
    if out.dtype != torch.int32 or out.numel() != m:
        raise ValueError("out must hold m int32 values")
    rp, rs = None, 0
    if recent is not None and n_recent:
        if recent.dtype != torch.int32 or recent.stride(-1) != 1:
            raise ValueError("recent must be int32 with unit stride along the tokens")
        rp, rs = recent.data_ptr(), recent.stride(0) if recent.dim() > 1 else 0
    _lib.ensure_init(logits.device.index or 0)
    _lib.check(_lib.load().zwg_llm_greedy(logits.data_ptr(), m, n_vocab, rp, rs, n_recent, window, float(penalty),
                                          out.data_ptr(), out.stride(0) if out.dim() else 1, _stream_of(logits)))
    return out


class LlmWeightsQ8:
    """A Qwen2 model's weights on the device (llm.Model / llm.Layer, src/llm.zig:15-60) and
    the zwg_llm_weights struct that points at them. `layers` is a list of dicts with keys
    attn_norm, wq, bq, wk, bk, wv, bv, wo, ffn_norm, w_gate, w_up, w_down; Q8 matrices are
    (q int8 [n][k], scales f32 [n][k/32]) pairs, the rest f32 vectors (biases may be None).
    Arrays may be numpy or torch; they are copied to `device` once."""

    Q8_KEYS = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")
    VEC_KEYS = ("attn_norm", "bq", "bk", "bv", "ffn_norm")

    def __init__(self, layers, embd, output, output_norm, eps: float, device: int = 0):
        torch = _torch()
        dev = torch.device("cuda", device)

        def t(a, dtype):
            if a is None:
                return None
            if not isinstance(a, torch.Tensor):
                a = torch.from_numpy(np.ascontiguousarray(a))
            return a.to(device=dev, dtype=dtype).contiguous()

        def q8(pair):
            return t(pair[0], torch.int8), t(pair[1], torch.float32)

        self.layers = []
        for L in layers:
            d = {k: q8(L[k]) for k in self.Q8_KEYS}
            d.update({k: t(L.get(k), torch.float32) for k in self.VEC_KEYS})
            self.layers.append(d)
        self.embd = q8(embd)
        self.output = self.embd if output is None else q8(output)
        self.output_norm = t(output_norm, torch.float32)
        self.eps = float(eps)
        self.n_vocab, self.n_embd = self.embd[0].shape
        self.n_ff = self.layers[0]["w_gate"][0].shape[0]
        self._c = None

    @staticmethod
    def _mat(pair):
        return _lib.Q8MatC(pair[0].data_ptr(), pair[1].data_ptr())

    def layer_c(self, i: int) -> _lib.LlmLayerWeightsC:
        L = self.layers[i]
        p = lambda a: a.data_ptr() if a is not None else None  # noqa: E731
        return _lib.LlmLayerWeightsC(p(L["attn_norm"]), self._mat(L["wq"]), self._mat(L["wk"]), self._mat(L["wv"]),
                                     self._mat(L["wo"]), p(L["bq"]), p(L["bk"]), p(L["bv"]), p(L["ffn_norm"]),
                                     self._mat(L["w_gate"]), self._mat(L["w_up"]), self._mat(L["w_down"]))

    def c_struct(self) -> _lib.LlmWeightsC:
        if self._c is None:
            arr = (_lib.LlmLayerWeightsC * len(self.layers))(*[self.layer_c(i) for i in range(len(self.layers))])
            self._arr = arr  # keeps the host array alive as long as the struct
            self._c = _lib.LlmWeightsC(self.n_vocab, self.n_embd, self.n_ff, self.eps, self._mat(self.embd),
                                       self._mat(self.output), self.output_norm.data_ptr(),
                                       ctypes.cast(arr, ctypes.POINTER(_lib.LlmLayerWeightsC)))
        return self._c



def layer_norm(x, w, b, eps: float = 1e-5, out=None):
    """ops.layerNorm (src/ops.zig:355-398) of the rows of a CUDA f32 [m][n] tensor."""
    torch = _torch()
    n = x.shape[-1]
    m = x.numel() // n
    out = torch.empty_like(x) if out is None else out
    _lib.ensure_init(x.device.index or 0)
    _lib.check(_lib.load().zwg_layer_norm(_dev_ptr(x, torch.float32, "x"), m, n, _dev_ptr(w, torch.float32, "w"),
                                          _dev_ptr(b, torch.float32, "b"), float(eps),
                                          _dev_ptr(out, torch.float32, "out"), _stream_of(x)))
    return out


def linear_q8_gelu(x, q, scales, bias=None, out=None):
    """gelu(x . W^T + b) with Q8 W (src/decoder.zig:197-198, ggml's tanh GELU)."""
    torch = _torch()
    m, k = x.shape
    q, sp = _q8_pair((q, scales), "w")
    n = q.shape[0]
    out = torch.empty(m, n, dtype=torch.float32, device=x.device) if out is None else out
    _lib.ensure_init(x.device.index or 0)
    _lib.check(_lib.load().zwg_linear_q8_gelu(_dev_ptr(x, torch.float32, "x"), m, k, q.data_ptr(), sp,
                                              _dev_ptr(bias, torch.float32, "bias") if bias is not None else None,
                                              n, _dev_ptr(out, torch.float32, "out"), _stream_of(x)))
    return out


class WhisperRules:
    """zwg_whisper_rules: the special token ids and options of Engine.sample
    (src/transcribe.zig:491-580). `hotwords` is a list of forms (token id lists), in the
    reference's order; they are copied to the device once."""

    def __init__(self, hotwords=(), hotword_bias: float = 5.0, max_initial_ts: float = 1.0, n_audio_ctx: int = 1500,
                 device: int = 0, **token_ids):
        torch = _torch()
        self.c = _lib.WhisperRulesC()
        _lib.check(_lib.load().zwg_whisper_rules_default(ctypes.byref(self.c)))
        for k, v in token_ids.items():
            setattr(self.c, k, int(v))
        self.c.n_audio_ctx = n_audio_ctx
        self.c.max_initial_ts = max_initial_ts
        self.c.hotword_bias = hotword_bias
        self._keep = []
        forms = [list(f) for f in hotwords]
        if forms:
            flat = [t for f in forms for t in f] or [0]
            offs = [0]
            for f in forms:
                offs.append(offs[-1] + len(f))
            d = torch.device("cuda", device)
            ht = torch.tensor(flat, dtype=torch.int32, device=d)
            ho = torch.tensor(offs, dtype=torch.int32, device=d)
            self._keep = [ht, ho]
            self.c.hotwords, self.c.hotword_offsets, self.c.n_hotwords = ht.data_ptr(), ho.data_ptr(), len(forms)


def whisper_sample(logits, tokens=None, n_tokens=None, has_ts=None, seek_delta=None, rules: WhisperRules = None):
    """Engine.sample (src/transcribe.zig:491-580) on each row of logits [n_batch][n_vocab]
    (CUDA f32, modified in place) with the device sampler (zwg_whisper_sample). tokens: CUDA
    int32 [n_batch][cap] with n_tokens [n_batch] of them sampled so far; has_ts, seek_delta:
    CUDA int32 [n_batch]. Returns (ids, tids), CUDA int32 [n_batch]."""
    torch = _torch()
    nb, nv = logits.shape
    rules = rules or WhisperRules(device=logits.device.index or 0)
    ids = torch.empty(nb, dtype=torch.int32, device=logits.device)
    tids = torch.empty_like(ids)
    tp = _dev_ptr(tokens, torch.int32, "tokens") if tokens is not None else None
    stride = tokens.shape[1] if tokens is not None else 0
    ntp = _dev_ptr(n_tokens, torch.int32, "n_tokens") if n_tokens is not None else None
    hp = _dev_ptr(has_ts, torch.int32, "has_ts") if has_ts is not None else None
    sp = _dev_ptr(seek_delta, torch.int32, "seek_delta") if seek_delta is not None else None
    _lib.check(_lib.load().zwg_whisper_sample(_dev_ptr(logits, torch.float32, "logits"), nb, nv, tp, stride, ntp, hp,
                                              sp, ctypes.byref(rules.c), ids.data_ptr(), tids.data_ptr(),
                                              _stream_of(logits)))
    return ids, tids


def whisper_decode_q8(state: "DecoderState", weights: "DecoderWeightsQ8", prompt, seek, seek_end,
                      rules: WhisperRules = None, n_max: int = 0, check_every: int = 8, scratch=None):
    """The token loop of one window per state window on the device (zwg_whisper_decode_q8):
    prompt CUDA int32 [n_batch][n_prompt]; seek, seek_end: per-window mel frames (lists).
    The cross K/V must be set. Returns one dict per window: tokens, tids, result_len,
    seek_delta, has_ts, failed."""
    torch = _torch()
    nb = state.n_batch
    dev = prompt.device
    rules = rules or WhisperRules(device=dev.index or 0)
    n_prompt = prompt.numel() // nb
    cap = n_max or (state.n_text_ctx // 2 - 4)
    win = torch.zeros(nb, 8, dtype=torch.int32, device=dev)
    win[:, 0] = torch.tensor(list(seek), dtype=torch.int32)
    win[:, 1] = torch.tensor(list(seek_end), dtype=torch.int32)
    tokens = torch.full((nb, cap), -1, dtype=torch.int32, device=dev)
    tids = torch.full((nb, cap), -1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    need = lib.zwg_whisper_decode_scratch_bytes(state._h, weights.n_vocab, n_prompt)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
    _lib.check(lib.zwg_whisper_decode_q8(state._h, ctypes.byref(weights.c_struct()), ctypes.byref(rules.c),
                                         _dev_ptr(prompt, torch.int32, "prompt"), n_prompt, n_max, win.data_ptr(),
                                         tokens.data_ptr(), tids.data_ptr(), cap, check_every, scratch.data_ptr(),
                                         scratch.numel(), _stream_of(prompt)))
    w = win.cpu().numpy()
    tk, td = tokens.cpu().numpy(), tids.cpu().numpy()
    out = []
    for b in range(nb):
        n = int(w[b, 2])
        out.append({"tokens": tk[b, :n].tolist(), "tids": td[b, :n].tolist(), "result_len": int(w[b, 5]),
                    "seek_delta": int(w[b, 3]), "has_ts": bool(w[b, 4]), "failed": bool(w[b, 6])})
    return out


class DecoderWeightsQ8:
    """The Whisper decoder's weights on the device (decoder.Decoder / decoder.Layer,
    src/decoder.zig:13-60) and the zwg_dec_weights struct that points at them. `tensors` maps
    the model file's names (decoder.token_embedding.weight, decoder.positional_embedding,
    decoder.ln.weight/bias, decoder.blocks.{i}.attn.query.weight, ...) to numpy or torch
    arrays (f16 or f32). The 2-d decoder matrices are quantized to Q8 on the device as the
    reference's loader does (Q8.quantize from the f16 values, src/decoder.zig:220-229); norms,
    biases and the position table stay f32."""

    ATTN = ("query", "key", "value", "out")

    def __init__(self, tensors, n_layer: int, device: int = 0):
        torch = _torch()
        dev = torch.device("cuda", device)
        _lib.ensure_init(device)

        def f32(name):
            a = tensors[name]
            if not isinstance(a, torch.Tensor):
                a = torch.from_numpy(np.ascontiguousarray(a))
            return a.to(device=dev, dtype=torch.float32).contiguous()

        def q8(name):
            return quantize_q8(f32(name))

        self.te = q8("decoder.token_embedding.weight")
        self.pe = f32("decoder.positional_embedding")
        self.ln_w, self.ln_b = f32("decoder.ln.weight"), f32("decoder.ln.bias")
        self.n_vocab, self.n_state = self.te[0].shape
        self.layers = []
        for i in range(n_layer):
            p = f"decoder.blocks.{i}."
            L = {
                "attn_ln_w": f32(p + "attn_ln.weight"), "attn_ln_b": f32(p + "attn_ln.bias"),
                "q": q8(p + "attn.query.weight"), "q_b": f32(p + "attn.query.bias"),
                "k": q8(p + "attn.key.weight"),
                "v": q8(p + "attn.value.weight"), "v_b": f32(p + "attn.value.bias"),
                "o": q8(p + "attn.out.weight"), "o_b": f32(p + "attn.out.bias"),
                "cross_ln_w": f32(p + "cross_attn_ln.weight"), "cross_ln_b": f32(p + "cross_attn_ln.bias"),
                "cq": q8(p + "cross_attn.query.weight"), "cq_b": f32(p + "cross_attn.query.bias"),
                "ck": q8(p + "cross_attn.key.weight"),
                "cv": q8(p + "cross_attn.value.weight"), "cv_b": f32(p + "cross_attn.value.bias"),
                "co": q8(p + "cross_attn.out.weight"), "co_b": f32(p + "cross_attn.out.bias"),
                "mlp_ln_w": f32(p + "mlp_ln.weight"), "mlp_ln_b": f32(p + "mlp_ln.bias"),
                "mlp0": q8(p + "mlp.0.weight"), "mlp0_b": f32(p + "mlp.0.bias"),
                "mlp1": q8(p + "mlp.2.weight"), "mlp1_b": f32(p + "mlp.2.bias"),
            }
            self.layers.append(L)
        self._c = None

    @staticmethod
    def _mat(pair):
        return _lib.Q8MatC(pair[0].data_ptr(), pair[1].data_ptr())

    def c_struct(self) -> _lib.DecWeightsC:
        if self._c is None:
            m = self._mat
            arr = (_lib.DecLayerWeightsC * len(self.layers))(*[
                _lib.DecLayerWeightsC(
                    L["attn_ln_w"].data_ptr(), L["attn_ln_b"].data_ptr(), m(L["q"]), L["q_b"].data_ptr(), m(L["k"]),
                    m(L["v"]), L["v_b"].data_ptr(), m(L["o"]), L["o_b"].data_ptr(), L["cross_ln_w"].data_ptr(),
                    L["cross_ln_b"].data_ptr(), m(L["cq"]), L["cq_b"].data_ptr(), m(L["ck"]), m(L["cv"]),
                    L["cv_b"].data_ptr(), m(L["co"]), L["co_b"].data_ptr(), L["mlp_ln_w"].data_ptr(),
                    L["mlp_ln_b"].data_ptr(), m(L["mlp0"]), L["mlp0_b"].data_ptr(), m(L["mlp1"]),
                    L["mlp1_b"].data_ptr())
                for L in self.layers])
            self._arr = arr  # keeps the host array alive as long as the struct
            self._c = _lib.DecWeightsC(self.n_vocab, m(self.te), self.pe.data_ptr(), self.ln_w.data_ptr(),
                                       self.ln_b.data_ptr(), ctypes.cast(arr, ctypes.POINTER(_lib.DecLayerWeightsC)))
        return self._c


# ---- Whisper encoder on the device (src/encoder.zig:118-179) -------------------------------

_GEMM_OUT = {"f32": 0, "f16": 1, "bf16": 2}


def gemm_f16(a, w, bias=None, gelu: bool = False, addend=None, accumulate: bool = False, out=None,
             out_dtype: str = "f32", M: int = None, K: int = None, lda: int = None, a_bs: int = None):
    """One f16 GEMM on the tensor cores (zwg_gemm_f16): out[b][m][n] = act(a[b][m] . w[n] +
    bias[n]) (+ addend[m][n]) (+ out when accumulate). a f16 [B][M][K] (or a strided view of
    rows given by M, K, lda, a_bs over a flat f16 buffer), w f16 [N][K]; out [B][M][N]."""
    torch = _torch()
    if a.dtype != torch.float16 or w.dtype != torch.float16:
        raise ValueError("a and w must be f16")
    N, Kw = w.shape
    if M is None:
        if a.dim() == 2:
            a = a.unsqueeze(0)
        B, M, K = a.shape
        lda, a_bs = K, M * K
    else:
        B = a.numel() // a_bs if a_bs else 1
        K = Kw if K is None else K
    dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[out_dtype]
    if out is None:
        out = torch.zeros(B, M, N, dtype=dt, device=a.device)
    _lib.ensure_init(a.device.index or 0)
    lib = _lib.load()
    rc = lib.zwg_gemm_f16(a.data_ptr(), lda, a_bs or 0, w.data_ptr(), Kw, M, N, K, B,
                          bias.data_ptr() if bias is not None else 0, 1 if gelu else 0,
                          addend.data_ptr() if addend is not None else 0, N if addend is not None else 0,
                          1 if accumulate else 0, out.data_ptr(), _GEMM_OUT[out_dtype], N, M * N, _stream_of(a))
    _lib.check(rc)
    return out


class EncoderWeightsF16:
    """The Whisper encoder's weights on the device (encoder.Encoder, src/encoder.zig:12-40)
    and the zwg_enc_weights struct that points at them. `tensors` maps the model file's names
    (encoder.conv1.weight [n_state][n_mels][3], encoder.positional_embedding,
    encoder.blocks.{i}.attn.query.weight, ...) to numpy or torch arrays. Matrices stay f16 (the
    file's values, exact); the convolution weights are stored tap-major ([n_out][3][n_in]) and
    the query/key/value rows stacked into one [3 n_state][n_state] matrix with the key's
    missing bias as zeros."""

    def __init__(self, tensors, n_layer: int, n_head: int, device: int = 0):
        torch = _torch()
        dev = torch.device("cuda", device)
        _lib.ensure_init(device)

        def t(name):
            a = tensors[name]
            if not isinstance(a, torch.Tensor):
                a = torch.from_numpy(np.ascontiguousarray(a))
            return a.to(device=dev)

        def f32(name):
            return t(name).to(torch.float32).contiguous()

        def f16(name):
            return t(name).to(torch.float16).contiguous()

        c1 = f16("encoder.conv1.weight")  # [n_state][n_mels][3]
        c2 = f16("encoder.conv2.weight")  # [n_state][n_state][3]
        self.n_state, self.n_mels = c1.shape[0], c1.shape[1]
        self.n_head, self.n_layer = n_head, n_layer
        self.conv1_w = c1.permute(0, 2, 1).contiguous().view(self.n_state, -1)
        self.conv2_w = c2.permute(0, 2, 1).contiguous().view(self.n_state, -1)
        self.conv1_b, self.conv2_b = f32("encoder.conv1.bias"), f32("encoder.conv2.bias")
        self.pos = f32("encoder.positional_embedding")
        self.n_ctx = self.pos.shape[0]
        self.ln_post_w, self.ln_post_b = f32("encoder.ln_post.weight"), f32("encoder.ln_post.bias")
        self.layers = []
        for i in range(n_layer):
            p = f"encoder.blocks.{i}."
            zeros = torch.zeros(self.n_state, dtype=torch.float32, device=dev)
            self.layers.append({
                "attn_ln_w": f32(p + "attn_ln.weight"), "attn_ln_b": f32(p + "attn_ln.bias"),
                "w_qkv": torch.cat([f16(p + "attn.query.weight"), f16(p + "attn.key.weight"),
                                    f16(p + "attn.value.weight")]).contiguous(),
                "b_qkv": torch.cat([f32(p + "attn.query.bias"), zeros, f32(p + "attn.value.bias")]).contiguous(),
                "w_o": f16(p + "attn.out.weight"), "b_o": f32(p + "attn.out.bias"),
                "mlp_ln_w": f32(p + "mlp_ln.weight"), "mlp_ln_b": f32(p + "mlp_ln.bias"),
                "w_mlp0": f16(p + "mlp.0.weight"), "b_mlp0": f32(p + "mlp.0.bias"),
                "w_mlp2": f16(p + "mlp.2.weight"), "b_mlp2": f32(p + "mlp.2.bias"),
            })
        self._c = None

    FIELDS = ("attn_ln_w", "attn_ln_b", "w_qkv", "b_qkv", "w_o", "b_o", "mlp_ln_w", "mlp_ln_b", "w_mlp0", "b_mlp0",
              "w_mlp2", "b_mlp2")

    def c_struct(self) -> _lib.EncWeightsC:
        if self._c is None:
            arr = (_lib.EncLayerWeightsC * len(self.layers))(*[
                _lib.EncLayerWeightsC(*[L[f].data_ptr() for f in self.FIELDS]) for L in self.layers])
            self._arr = arr  # keeps the host array alive as long as the struct
            self._c = _lib.EncWeightsC(self.n_mels, self.n_ctx, self.n_state, self.n_head, self.n_layer,
                                       self.conv1_w.data_ptr(), self.conv1_b.data_ptr(), self.conv2_w.data_ptr(),
                                       self.conv2_b.data_ptr(), self.pos.data_ptr(),
                                       ctypes.cast(arr, ctypes.POINTER(_lib.EncLayerWeightsC)),
                                       self.ln_post_w.data_ptr(), self.ln_post_b.data_ptr())
        return self._c

    def scratch_bytes(self, n_windows: int) -> int:
        return int(_lib.load().zwg_enc_scratch_bytes(ctypes.byref(self.c_struct()), n_windows))


def encoder_forward(weights: EncoderWeightsF16, mel, n_windows: int, offsets=None, out=None, scratch=None):
    """Encoder.forward (src/encoder.zig:118-179) for n_windows windows of the device mel
    [n_mels][n_len] f32 (zwg_enc_forward_f16): window i starts at frame offsets[i] (a CUDA int32
    tensor) or i * 2 n_ctx. Returns out [n_windows][n_ctx][n_state] f32."""
    torch = _torch()
    _dev_ptr(mel, torch.float32, "mel")
    n_len = mel.shape[1]
    if out is None:
        out = torch.empty(n_windows, weights.n_ctx, weights.n_state, dtype=torch.float32, device=mel.device)
    need = weights.scratch_bytes(n_windows)
    if scratch is None:
        scratch = torch.empty(max(need, 256), dtype=torch.uint8, device=mel.device)
    off = _dev_ptr(offsets, torch.int32, "offsets") if offsets is not None else 0
    rc = _lib.load().zwg_enc_forward_f16(ctypes.byref(weights.c_struct()), mel.data_ptr(), n_len, off, n_windows,
                                         out.data_ptr(), scratch.data_ptr(), scratch.numel(), _stream_of(mel))
    _lib.check(rc)
    return out


def log_mel(samples, filters, out=None):
    """mel.logMel (src/mel.zig:103-157) on the device (zwg_log_mel): samples [n] f32 CUDA
    tensor at 16 kHz, filters [n_mel][201] f32; returns [n_mel][n_len] f32."""
    torch = _torch()
    _dev_ptr(samples, torch.float32, "samples")
    _dev_ptr(filters, torch.float32, "filters")
    lib = _lib.load()
    _lib.ensure_init(samples.device.index or 0)
    n = samples.numel()
    n_mel = filters.shape[0]
    n_len = int(lib.zwg_mel_frames(n))
    if out is None:
        out = torch.empty(n_mel, n_len, dtype=torch.float32, device=samples.device)
    scratch = torch.empty(int(lib.zwg_mel_scratch_bytes()), dtype=torch.uint8, device=samples.device)
    _lib.check(lib.zwg_log_mel(samples.data_ptr(), n, filters.data_ptr(), n_mel, out.data_ptr(), scratch.data_ptr(),
                               scratch.numel(), _stream_of(samples)))
    return out
