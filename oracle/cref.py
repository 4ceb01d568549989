"""Loader for the C restatement of the reference attention (oracle/attn_ref.c).

TEST INFRASTRUCTURE ONLY: used by tests (as a cross-check) and by bench.py's
`cpu_baseline` and `--impl reference` legs (as the timed CPU baseline).

Two builds ship: AVX-512 (16 lanes, the reference's width on such hosts) and AVX2
(8 lanes). The loader picks the widest one the running CPU supports.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "attn_ref.c")
LIBS = {
    "avx512": os.path.join(HERE, "libattn_ref_avx512.so"),
    "avx2": os.path.join(HERE, "libattn_ref_avx2.so"),
}
FLAGS = {
    "avx512": ["-mavx512f", "-mavx2", "-mfma"],
    "avx2": ["-mavx2", "-mfma"],
}


class Shape(ctypes.Structure):
    _fields_ = [
        ("n_q", ctypes.c_size_t), ("n_kv", ctypes.c_size_t), ("n_head", ctypes.c_size_t),
        ("n_head_kv", ctypes.c_size_t), ("d", ctypes.c_size_t), ("q_stride", ctypes.c_size_t),
        ("kv_stride", ctypes.c_size_t), ("out_stride", ctypes.c_size_t), ("causal", ctypes.c_int),
        ("kt_stride", ctypes.c_size_t),
    ]


def build(force: bool = False) -> None:
    for isa, path in LIBS.items():
        if not force and os.path.exists(path) and os.path.getmtime(path) >= os.path.getmtime(SRC):
            continue
        cmd = ["gcc", "-O3", "-fPIC", "-shared", "-fopenmp", *FLAGS[isa], SRC, "-o", path, "-lm"]
        subprocess.check_call(cmd)


def _cpu_flags() -> set:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


_lib = None
_isa = None


def load():
    global _lib, _isa
    if _lib is not None:
        return _lib
    flags = _cpu_flags()
    isa = "avx512" if "avx512f" in flags else "avx2"
    path = LIBS[isa]
    if not os.path.exists(path):
        build()
    lib = ctypes.CDLL(path)
    lib.zwref_attention_ex.restype = ctypes.c_int
    lib.zwref_attention_ex.argtypes = [ctypes.POINTER(Shape)] + [ctypes.c_void_p] * 5 + [ctypes.c_int]
    lib.zwref_scratch_floats.restype = ctypes.c_size_t
    lib.zwref_scratch_floats.argtypes = [ctypes.POINTER(Shape)]
    lib.zwref_vector_width.restype = ctypes.c_size_t
    _lib, _isa = lib, isa
    return lib


def isa() -> str:
    load()
    return _isa


def make_shape(sh) -> Shape:
    return Shape(sh.n_q, sh.n_kv, sh.n_head, sh.n_head_kv, sh.d, sh.q_stride, sh.kv_stride,
                 sh.out_stride, 1 if sh.causal else 0, sh.kt_stride or 0)


class Runner:
    """Holds scratch for repeated calls with one shape (the reference sizes scratch once
    per model, encoder.zig:100 / decoder.zig:137-140 / llm.zig:147)."""

    def __init__(self, sh, n_threads: int = 0):
        self.lib = load()
        self.sh = make_shape(sh)
        self.n_threads = n_threads
        self.scratch = np.empty(max(1, self.lib.zwref_scratch_floats(ctypes.byref(self.sh))), np.float32)

    def __call__(self, q, k, v, out):
        rc = self.lib.zwref_attention_ex(ctypes.byref(self.sh), q.ctypes.data, k.ctypes.data,
                                         v.ctypes.data, self.scratch.ctypes.data, out.ctypes.data,
                                         self.n_threads)
        if rc != 0:
            raise ValueError("attn_ref rejected the shape")
        return out


def attention_ex(q, k, v, sh, out=None, n_threads: int = 0):
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    if out is None:
        out = np.zeros(max(sh.n_q, 1) * sh.out_stride, np.float32)
    return Runner(sh, n_threads)(q, k, v, out)
