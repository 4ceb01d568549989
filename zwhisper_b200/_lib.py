"""ctypes binding of libzwgpu.so (include/zwgpu.h).

The library is required: importing the bindings raises if it is missing, so no caller
can silently run without the CUDA path.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libzwgpu.so")

ZWG_OK = 0
ZWG_ERROR = 2
ZWG_TIMEOUT = 4
ZWG_MATH_F32 = 0
ZWG_MATH_BF16 = 1
ZWG_MATH_TF32 = 2

c_size = ctypes.c_size_t
c_ptr = ctypes.c_void_p


class WhisperRulesC(ctypes.Structure):
    """zwg_whisper_rules: the special token ids and options of Engine.sample
    (src/transcribe.zig:491-580, src/model.zig:37-47); hotword arrays are device pointers."""

    _fields_ = [
        ("eot", ctypes.c_int32), ("sot", ctypes.c_int32), ("translate", ctypes.c_int32),
        ("transcribe", ctypes.c_int32), ("solm", ctypes.c_int32), ("prev", ctypes.c_int32),
        ("nosp", ctypes.c_int32), ("not_", ctypes.c_int32), ("beg", ctypes.c_int32), ("space", ctypes.c_int32),
        ("n_audio_ctx", ctypes.c_int32), ("max_initial_ts", ctypes.c_float), ("hotword_bias", ctypes.c_float),
        ("hotwords", c_ptr), ("hotword_offsets", c_ptr), ("n_hotwords", ctypes.c_int32),
    ]


class WhisperWindowC(ctypes.Structure):
    """zwg_whisper_window: one window's state in the token loop (src/transcribe.zig:292-365)."""

    _fields_ = [(n, ctypes.c_int32) for n in ("seek", "seek_end", "n_tokens", "seek_delta", "has_ts", "result_len",
                                               "failed", "done")]


class AttnShapeC(ctypes.Structure):
    """zwg_attn_shape (include/zwgpu.h), the C mirror of AttnShape (src/ops.zig:477-492)."""

    _fields_ = [
        ("n_q", c_size), ("n_kv", c_size), ("n_head", c_size), ("n_head_kv", c_size), ("d", c_size),
        ("q_stride", c_size), ("kv_stride", c_size), ("out_stride", c_size), ("causal", ctypes.c_int32),
        ("kt_stride", c_size),
    ]


class BatchC(ctypes.Structure):
    """zwg_batch (include/zwgpu.h)."""

    _fields_ = [
        ("n_batch", c_size), ("q_batch_stride", c_size), ("k_batch_stride", c_size),
        ("v_batch_stride", c_size), ("out_batch_stride", c_size),
    ]


class Q8MatC(ctypes.Structure):
    """zwg_q8_mat: int8 [n][k] and f32 scales [n][k/32] on the device (gemm.Q8)."""

    _fields_ = [("q", c_ptr), ("scales", c_ptr)]


class LlmLayerWeightsC(ctypes.Structure):
    """zwg_llm_layer_weights (llm.Layer, src/llm.zig:15-30, without the caches)."""

    _fields_ = [
        ("attn_norm", c_ptr), ("wq", Q8MatC), ("wk", Q8MatC), ("wv", Q8MatC), ("wo", Q8MatC),
        ("bq", c_ptr), ("bk", c_ptr), ("bv", c_ptr), ("ffn_norm", c_ptr),
        ("w_gate", Q8MatC), ("w_up", Q8MatC), ("w_down", Q8MatC),
    ]


class LlmWeightsC(ctypes.Structure):
    """zwg_llm_weights (llm.Model's weights, src/llm.zig:32-60)."""

    _fields_ = [
        ("n_vocab", c_size), ("n_embd", c_size), ("n_ff", c_size), ("eps", ctypes.c_float),
        ("embd", Q8MatC), ("output", Q8MatC), ("output_norm", c_ptr),
        ("layers", ctypes.POINTER(LlmLayerWeightsC)),
    ]


class DecLayerWeightsC(ctypes.Structure):
    """zwg_dec_layer_weights (decoder.Layer, src/decoder.zig:13-43, without the state)."""

    _fields_ = [
        ("attn_ln_w", c_ptr), ("attn_ln_b", c_ptr), ("q", Q8MatC), ("q_b", c_ptr), ("k", Q8MatC), ("v", Q8MatC),
        ("v_b", c_ptr), ("o", Q8MatC), ("o_b", c_ptr), ("cross_ln_w", c_ptr), ("cross_ln_b", c_ptr),
        ("cq", Q8MatC), ("cq_b", c_ptr), ("ck", Q8MatC), ("cv", Q8MatC), ("cv_b", c_ptr), ("co", Q8MatC),
        ("co_b", c_ptr), ("mlp_ln_w", c_ptr), ("mlp_ln_b", c_ptr), ("mlp0", Q8MatC), ("mlp0_b", c_ptr),
        ("mlp1", Q8MatC), ("mlp1_b", c_ptr),
    ]


class DecWeightsC(ctypes.Structure):
    """zwg_dec_weights (decoder.Decoder's weights, src/decoder.zig:45-60)."""

    _fields_ = [
        ("n_vocab", c_size), ("te", Q8MatC), ("pe", c_ptr), ("ln_w", c_ptr), ("ln_b", c_ptr),
        ("layers", ctypes.POINTER(DecLayerWeightsC)),
    ]


class EncLayerWeightsC(ctypes.Structure):
    """zwg_enc_layer_weights (encoder.Block, src/encoder.zig:12-30): f16 matrices, f32 vectors."""

    _fields_ = [
        ("attn_ln_w", c_ptr), ("attn_ln_b", c_ptr), ("w_qkv", c_ptr), ("b_qkv", c_ptr), ("w_o", c_ptr),
        ("b_o", c_ptr), ("mlp_ln_w", c_ptr), ("mlp_ln_b", c_ptr), ("w_mlp0", c_ptr), ("b_mlp0", c_ptr),
        ("w_mlp2", c_ptr), ("b_mlp2", c_ptr),
    ]


class EncWeightsC(ctypes.Structure):
    """zwg_enc_weights (encoder.Encoder's weights, src/encoder.zig:32-40)."""

    _fields_ = [
        ("n_mels", c_size), ("n_ctx", c_size), ("n_state", c_size), ("n_head", c_size), ("n_layer", c_size),
        ("conv1_w", c_ptr), ("conv1_b", c_ptr), ("conv2_w", c_ptr), ("conv2_b", c_ptr), ("pos", c_ptr),
        ("layers", ctypes.POINTER(EncLayerWeightsC)), ("ln_post_w", c_ptr), ("ln_post_b", c_ptr),
    ]


# name -> (restype, argtypes); every symbol include/zwgpu.h declares
SIGNATURES = {
    "zwg_version": (ctypes.c_int, []),
    "zwg_init": (ctypes.c_int, [ctypes.c_int]),
    "zwg_shutdown": (ctypes.c_int, []),
    "zwg_last_error": (c_size, [ctypes.c_char_p, c_size]),
    "zwg_device_count": (ctypes.c_int, []),
    "zwg_attention": (ctypes.c_int, [ctypes.POINTER(AttnShapeC), c_ptr, c_ptr, c_ptr, c_ptr]),
    "zwg_attention_mha": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_size, c_size, c_size, c_size, ctypes.c_int32, c_ptr]),
    "zwg_attention_batch_host": (ctypes.c_int, [ctypes.POINTER(AttnShapeC), ctypes.POINTER(BatchC), c_ptr, c_ptr,
                                                c_ptr, c_ptr]),
    "zwg_attention_workspace": (c_size, [ctypes.POINTER(AttnShapeC), ctypes.POINTER(BatchC)]),
    "zwg_attention_dev": (ctypes.c_int, [ctypes.POINTER(AttnShapeC), ctypes.POINTER(BatchC), c_ptr, c_ptr, c_ptr,
                                         c_ptr, c_ptr, c_size, c_ptr]),
    "zwg_attention_dev_noalloc": (ctypes.c_int, [ctypes.POINTER(AttnShapeC), ctypes.POINTER(BatchC), c_ptr, c_ptr,
                                                 c_ptr, c_ptr, c_ptr]),
    "zwg_enc_attn_bf16": (ctypes.c_int, [c_size, c_size, c_size, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "zwg_f32_to_bf16": (ctypes.c_int, [c_ptr, c_ptr, c_size, c_ptr]),
    "zwg_rope_kt_append": (ctypes.c_int, [c_size, c_size, c_size, c_size, c_size, c_size, c_size, c_ptr, c_ptr,
                                          c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_size, c_size, c_size, c_ptr]),
    "zwg_sync": (ctypes.c_int, []),
    "zwg_set_math": (ctypes.c_int, [ctypes.c_int]),
    "zwg_selftest_timeout": (ctypes.c_int, []),
    "zwg_q8_quantize": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, c_ptr]),
    "zwg_linear_q8": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, c_ptr, c_size, c_ptr, c_ptr]),
    "zwg_q8_tensor_cores": (ctypes.c_int, [ctypes.c_int]),
    "zwg_dec_state_create": (ctypes.c_int, [c_size, c_size, c_size, c_size, c_size, c_size, ctypes.POINTER(c_ptr)]),
    "zwg_dec_state_destroy": (ctypes.c_int, [c_ptr]),
    "zwg_dec_state_cache": (ctypes.c_int, [c_ptr, c_size, ctypes.POINTER(c_ptr), ctypes.POINTER(c_ptr),
                                           ctypes.POINTER(c_ptr), ctypes.POINTER(c_ptr)]),
    "zwg_cross_kv_set": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, c_ptr]),
    "zwg_dec_step_attn": (ctypes.c_int, [c_ptr, c_size, ctypes.c_int, c_ptr, c_ptr, c_ptr, c_size, c_size, c_ptr,
                                         c_ptr]),
    "zwg_llm_state_create": (ctypes.c_int, [c_size, c_size, c_size, c_size, c_size, c_size, ctypes.c_double,
                                            ctypes.POINTER(c_ptr)]),
    "zwg_llm_state_destroy": (ctypes.c_int, [c_ptr]),
    "zwg_llm_state_cache": (ctypes.c_int, [c_ptr, c_size, ctypes.POINTER(c_ptr), ctypes.POINTER(c_ptr)]),
    "zwg_llm_append_rope": (ctypes.c_int, [c_ptr, c_size, c_ptr, c_ptr, c_ptr, c_size, c_size, c_ptr]),
    "zwg_llm_attn_prefill": (ctypes.c_int, [c_ptr, c_size, c_ptr, c_size, c_size, c_ptr, c_ptr]),
    "zwg_llm_attn_decode": (ctypes.c_int, [c_ptr, c_size, c_ptr, c_size, c_ptr, c_ptr]),
    "zwg_rms_norm": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, ctypes.c_float, c_ptr, c_ptr]),
    "zwg_linear_q8_add": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, c_size, c_ptr, c_ptr]),
    "zwg_linear_q8_silu_mul": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, c_ptr, c_ptr, c_size, c_ptr,
                                              c_ptr]),
    "zwg_embed_q8": (ctypes.c_int, [c_ptr, c_size, c_ptr, c_ptr, c_size, c_size, c_ptr, c_ptr]),
    "zwg_llm_greedy": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_size, c_size, c_size, ctypes.c_float, c_ptr,
                                      c_size, c_ptr]),
    "zwg_llm_qkv_q8": (ctypes.c_int, [c_ptr, c_size, c_ptr, ctypes.POINTER(LlmLayerWeightsC), c_size, c_size, c_ptr,
                                      c_ptr]),
    "zwg_llm_scratch_bytes": (c_size, [c_ptr, c_size, c_size]),
    "zwg_llm_layer_q8": (ctypes.c_int, [c_ptr, c_size, ctypes.POINTER(LlmWeightsC), c_ptr, c_size, c_size, c_ptr,
                                        c_size, c_ptr]),
    "zwg_llm_forward_q8": (ctypes.c_int, [c_ptr, ctypes.POINTER(LlmWeightsC), c_ptr, c_size, c_size, c_ptr, c_ptr,
                                          c_ptr, c_size, c_ptr]),
    "zwg_layer_norm": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, ctypes.c_float, c_ptr, c_ptr]),
    "zwg_linear_q8_gelu": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, c_ptr, c_size, c_ptr, c_ptr]),
    "zwg_dec_set_audio_q8": (ctypes.c_int, [c_ptr, ctypes.POINTER(DecWeightsC), c_size, c_ptr, c_ptr]),
    "zwg_dec_scratch_bytes": (c_size, [c_ptr, c_size]),
    "zwg_whisper_rules_default": (ctypes.c_int, [ctypes.POINTER(WhisperRulesC)]),
    "zwg_whisper_sample": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_size, c_ptr, c_ptr, c_ptr,
                                          ctypes.POINTER(WhisperRulesC), c_ptr, c_ptr, c_ptr]),
    "zwg_whisper_window_init": (ctypes.c_int, [c_ptr, c_size, ctypes.POINTER(WhisperRulesC), c_ptr]),
    "zwg_whisper_step": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_ptr, c_ptr, c_size,
                                        ctypes.POINTER(WhisperRulesC), c_size, c_ptr, c_ptr]),
    "zwg_whisper_decode_scratch_bytes": (c_size, [c_ptr, c_size, c_size]),
    "zwg_whisper_decode_q8": (ctypes.c_int, [c_ptr, ctypes.POINTER(DecWeightsC), ctypes.POINTER(WhisperRulesC), c_ptr,
                                             c_size, c_size, c_ptr, c_ptr, c_ptr, c_size, c_size, c_ptr, c_size,
                                             c_ptr]),
    "zwg_enc_scratch_bytes": (c_size, [ctypes.POINTER(EncWeightsC), c_size]),
    "zwg_mel_frames": (c_size, [c_size]),
    "zwg_mel_scratch_bytes": (c_size, []),
    "zwg_log_mel": (ctypes.c_int, [c_ptr, c_size, c_ptr, c_size, c_ptr, c_ptr, c_size, c_ptr]),
    "zwg_enc_forward_f16": (ctypes.c_int, [ctypes.POINTER(EncWeightsC), c_ptr, c_size, c_ptr, c_size, c_ptr, c_ptr,
                                           c_size, c_ptr]),
    "zwg_gemm_f16": (ctypes.c_int, [c_ptr, c_size, c_size, c_ptr, c_size, c_size, c_size, c_size, c_size, c_ptr,
                                    ctypes.c_int, c_ptr, c_size, ctypes.c_int, c_ptr, ctypes.c_int, c_size, c_size,
                                    c_ptr]),
    "zwg_dec_forward_q8": (ctypes.c_int, [c_ptr, ctypes.POINTER(DecWeightsC), c_ptr, c_size, c_size, c_ptr, c_ptr,
                                          c_ptr, c_size, c_ptr]),
}

ZWG_DEC_SELF = 0
ZWG_DEC_CROSS = 1

_lib = None
_lock = threading.Lock()


class ZwgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"zwgpu error {code}: {msg}")
        self.code = code


def load():
    """Load libzwgpu.so; raise if it is missing (no fallback path exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m zwhisper_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(512)
    lib.zwg_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != ZWG_OK:
        raise ZwgError(rc, last_error())


_bound = threading.local()


def ensure_init(device: int) -> None:
    """Bind the calling thread to `device` (zwg_init), once per thread and device."""
    lib = load()
    if getattr(_bound, "device", None) != device:
        check(lib.zwg_init(device))
        _bound.device = device
