"""Multi-GPU sharding logic on the CPU: contiguous blocks, the max-over-ranks timing
reduction on a world-size-2 gloo group, and the in-process runner's re-queueing of a
failed device's block (failure made on the host: a worker that raises)."""
import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from zwhisper_b200.shard import ShardRunner, max_over_ranks, shard_range


def test_shard_range_partitions():
    for n in (0, 1, 7, 64):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                s, e = shard_range(n, r, world)
                assert 0 <= s <= e <= n
                seen.extend(range(s, e))
            assert seen == list(range(n))
            sizes = [shard_range(n, r, world)[1] - shard_range(n, r, world)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    import torch.distributed as dist

    from oracle import attention as A
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    # each rank takes its block of 6 windows of a small attention problem
    rng = np.random.default_rng(0)
    n_win, n_ctx, ns, H = 6, 20, 64, 2
    q_all = rng.standard_normal((n_win, n_ctx * ns), dtype=np.float32)
    k_all = rng.standard_normal((n_win, n_ctx * ns), dtype=np.float32)
    v_all = rng.standard_normal((n_win, n_ctx * ns), dtype=np.float32)
    s, e = shard_range(n_win, rank, world)
    outs = {i: A.attention(q_all[i], k_all[i], v_all[i], n_ctx, n_ctx, ns, H, False) for i in range(s, e)}
    t = max_over_ranks(float(rank + 1) * 0.5, world)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, t, {i: o.tolist() for i, o in outs.items()}))


def test_two_rank_gloo_shards_and_timing_reduction():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import attention as A
    rng = np.random.default_rng(0)
    n_win, n_ctx, ns, H = 6, 20, 64, 2
    q_all = rng.standard_normal((n_win, n_ctx * ns), dtype=np.float32)
    k_all = rng.standard_normal((n_win, n_ctx * ns), dtype=np.float32)
    v_all = rng.standard_normal((n_win, n_ctx * ns), dtype=np.float32)
    merged = {}
    for rank, t, outs in results:
        assert t == 1.0  # max over ranks of (rank + 1) * 0.5
        merged.update(outs)
    assert sorted(merged) == list(range(n_win))
    for i in range(n_win):
        want = A.attention(q_all[i], k_all[i], v_all[i], n_ctx, n_ctx, ns, H, False)
        np.testing.assert_array_equal(np.array(merged[i], np.float32), want)


def test_runner_requeues_failed_device_block():
    calls = []

    def fn(dev, s, e):
        calls.append((dev, s, e))
        if dev == 1:
            raise RuntimeError("injected launch failure")
        time.sleep(0.05)  # healthy devices are busy long enough for device 1 to take a block
        return list(range(s, e))

    res = ShardRunner([0, 1, 2]).run(fn, 30, blocks=6)
    assert [x for block in res.outputs for x in block] == list(range(30))
    assert 1 in res.failures and "injected" in res.failures[1]
    assert all(dev != 1 for dev in res.placement.values())


def test_runner_bind_failure_and_total_failure():
    def bind(dev):
        if dev == 0:
            raise RuntimeError("no such device")

    res = ShardRunner([0, 1], bind=bind).run(lambda d, s, e: (d, s, e), 10)
    assert res.failures[0].startswith("bind")
    assert all(v == 1 for v in res.placement.values())

    def always_fail(dev, s, e):
        raise RuntimeError("down")

    with pytest.raises(RuntimeError):
        ShardRunner([0, 1]).run(always_fail, 4)
