"""The C-ABI library on a host without a GPU: it loads, exports every symbol that
include/zwgpu.h declares, and fails cleanly (status 2 with a message, no abort) where a
device is needed. No compute call is made here."""
import ctypes
import os
import re
import subprocess

import pytest

from tests.conftest import ROOT, has_gpu

HEADER = os.path.join(ROOT, "include", "zwgpu.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"ZWG_API\s+(?:int|size_t)\s+(zwg_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ["zwg_init", "zwg_attention", "zwg_attention_dev", "zwg_enc_attn_bf16", "zwg_rope_kt_append"]:
        assert name in syms


def test_library_loads_and_exports_every_declared_symbol():
    from zwhisper_b200 import _lib
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(zwg_\w+)", out))
    assert exported == set(declared_symbols())


def test_no_device_paths_fail_cleanly():
    if has_gpu():
        pytest.skip("a GPU is present")
    from zwhisper_b200 import _lib
    lib = _lib.load()
    assert lib.zwg_version() == 1
    assert lib.zwg_device_count() == 0
    assert lib.zwg_init(0) == _lib.ZWG_ERROR
    assert "not available" in _lib.last_error()
    # a compute entry point without a context reports status 2, it does not crash
    sh = _lib.AttnShapeC(1, 1, 1, 1, 64, 64, 64, 64, 0, 0)
    assert lib.zwg_attention(ctypes.byref(sh), None, None, None, None) == _lib.ZWG_ERROR
    assert "zwg_init" in _lib.last_error()


def test_missing_library_raises(tmp_path, monkeypatch):
    from zwhisper_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "libzwgpu.so"))
    with pytest.raises(ImportError):
        _lib.load()


def test_workspace_sizer_and_shape_mirror():
    from zwhisper_b200 import ops
    sh = ops.mha_shape(1, 1500, 512, 8, False)
    assert sh.d == 64 and sh.q_stride == 512
    assert sh.extents() == (512, 1500 * 512, 1500 * 512, 512)
    # one query row per kv head: the split-K path, partials need workspace
    assert ops.attention_workspace_bytes(sh, 32) > 0
    # a prefill-sized call runs the tiled kernel without workspace
    assert ops.attention_workspace_bytes(ops.mha_shape(256, 1500, 512, 8, False), 1) == 0
    kt = ops.AttnShape(1, 2001, 14, 2, 64, 896, 128, 896, True, 2048)
    assert kt.extents()[1] == 2 * 64 * 2048
    with pytest.raises(ValueError):
        ops.mha_shape(1, 1, 100, 3, False)
