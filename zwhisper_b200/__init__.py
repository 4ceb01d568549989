"""zwhisper_b200: a B200 (sm_100a) attention engine for zwhisper.

The product is libzwgpu.so (C ABI, include/zwgpu.h), built from csrc/ with nvcc. This
package holds the build step, the ctypes binding and a host-side mirror of the reference's
attention operator interface (`ops`), plus the multi-GPU shard runner (`shard`).
"""
from . import _lib  # noqa: F401

__all__ = ["ops"]
