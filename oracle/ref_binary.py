"""The reference's own shipped binary as a timed CPU baseline (test and benchmark
infrastructure; nothing in the product runs it).

The reference's Zig source cannot be built here (no Zig toolchain), but its tree ships a
prebuilt executable, zig-out-safe/bin/zwhisper. `copy_from` copies it, unchanged, into
oracle/_ref/ (kept out of git, but shipped with the repository to the GPU box), where
`bench_attention` runs its `bench <threads>` command (src/bench.zig:50-77) and reads the
"enc attention 1500x1500 x8 heads" line: the reference's CPU attention on the base.en
encoder shape (8 heads of d 64 over 1500 frames, 4 * 1500^2 * 512 FLOP per call). The
binary is only executed, never inspected.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
BINARY = os.path.join(REF_DIR, "zwhisper")
ATTN_FLOP = 4 * 1500 * 1500 * 512   # one call of the bench's attention shape


def copy_from(ref_root: str) -> Optional[str]:
    """Copy the shipped binary into oracle/_ref/ when the reference tree is present."""
    src = os.path.join(ref_root, "zig-out-safe", "bin", "zwhisper")
    if not os.path.isfile(src):
        return None
    os.makedirs(REF_DIR, exist_ok=True)
    if not os.path.exists(BINARY) or os.path.getmtime(BINARY) < os.path.getmtime(src):
        shutil.copy2(src, BINARY)
    return BINARY


def bench_attention(threads: int, timeout: float = 120.0) -> Optional[dict]:
    """The binary's `bench <threads>` attention line: ms per call and GFLOP/s; None when the
    binary is absent or cannot run on this host."""
    if not os.path.isfile(BINARY):
        return None
    try:
        r = subprocess.run([BINARY, "bench", str(threads)], capture_output=True, text=True, timeout=timeout)
    except (OSError, subprocess.SubprocessError):
        return None
    if r.returncode != 0:
        return None
    for line in r.stdout.splitlines():
        if line.startswith("enc attention"):
            m = re.search(r"([0-9.]+)\s*ms\s+([0-9.]+)\s*GFLOP/s", line)
            if m:
                return {"ms": float(m.group(1)), "gflops": float(m.group(2)), "threads": threads, "line": line.strip()}
    return None
