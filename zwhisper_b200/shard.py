"""Sharding independent windows or sequences over GPUs (no collective on the data path).

Whisper's 30 s windows and the LLM's sequences are independent units: each one's
encoder output, cross K/V and KV cache are private (src/transcribe.zig:276-396 advances
windows one by one; src/llm.zig keeps one cache per model). So the units are split into
contiguous blocks, one per GPU, and results are gathered on the host.

Two ways to run:
  - one process per GPU (torch.distributed.run; `shard_range` + `max_over_ranks`, which is
    what bench.py does; the only collectives are a barrier and the timing reduction);
  - one process, one host thread per GPU (`ShardRunner`), each thread bound to its device
    context with zwg_init. If a device's block fails, the block is re-queued on the devices
    that are still healthy, and the failure is reported in the result.
"""
from __future__ import annotations

import queue
import threading
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous block [start, end) of n units for `rank` of `world` (sizes differ by at
    most one; every unit belongs to exactly one rank)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    return n * rank // world, n * (rank + 1) // world


def max_over_ranks(x: float, world: int, device=None) -> float:
    """Max of a per-rank scalar (a timing) over the process group; identity at world 1.
    Works on gloo (CPU) and nccl (GPU) groups."""
    if world == 1:
        return float(x)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


@dataclass
class ShardResult:
    outputs: List[Any]
    failures: Dict[int, str] = field(default_factory=dict)  # device -> error text
    placement: Dict[int, int] = field(default_factory=dict)  # block index -> device that ran it


class ShardRunner:
    """Run fn(device, start, end) over contiguous blocks of n units, one host thread per
    device. `bind(device)` runs once in each thread before its first block (zwg_init for
    the real engine). A block whose call raises is re-queued for another device; a device
    that failed takes no further blocks. If every device fails, RuntimeError is raised."""

    def __init__(self, devices: Sequence[int], bind: Optional[Callable[[int], None]] = None):
        if not devices:
            raise ValueError("no devices")
        self.devices = list(devices)
        self.bind = bind

    def run(self, fn: Callable[[int, int, int], Any], n: int, blocks: Optional[int] = None) -> ShardResult:
        nb = blocks or len(self.devices)
        ranges = [shard_range(n, i, nb) for i in range(nb)]
        work: "queue.Queue[int]" = queue.Queue()
        for i in range(nb):
            work.put(i)
        outputs: List[Any] = [None] * nb
        done = [False] * nb
        res = ShardResult(outputs)
        lock = threading.Lock()
        healthy = set(self.devices)

        def worker(dev: int):
            try:
                if self.bind:
                    self.bind(dev)
            except Exception as e:  # device unusable: leave its blocks to the others
                with lock:
                    res.failures[dev] = f"bind: {e}"
                    healthy.discard(dev)
                return
            while True:
                with lock:
                    if all(done) or dev not in healthy:
                        return
                try:
                    i = work.get(timeout=0.05)
                except queue.Empty:
                    with lock:
                        if all(done) or not healthy:
                            return
                    continue
                s, e = ranges[i]
                try:
                    out = fn(dev, s, e)
                except Exception as exc:
                    with lock:
                        res.failures[dev] = str(exc)
                        healthy.discard(dev)
                    work.put(i)
                    return
                with lock:
                    outputs[i] = out
                    done[i] = True
                    res.placement[i] = dev

        threads = [threading.Thread(target=worker, args=(d,), daemon=True) for d in self.devices]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if not all(done):
            raise RuntimeError(f"shards left unprocessed; device failures: {res.failures}")
        return res
