"""Batch sharding across ranks, on the CPU with two gloo processes.

What bench.py does on N GPUs: every rank regenerates the whole batch's prompts
from the seed, keeps its contiguous shard, works on it with no data exchange,
and only the timing (and here the shard contents) are gathered. The test checks
that the shards partition the batch exactly, that each rank's prompts equal
the corresponding rows of the full batch, and that a max-over-ranks reduction
of per-rank times (how bench.py reports a multi-GPU step) picks the slowest.
"""
import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from tie_b200 import synth
from tie_b200.shard import shard_range


def test_shard_range_partitions():
    for n in (1, 7, 8, 64, 256, 257):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                s, k = shard_range(n, r, world)
                covered += list(range(s, s + k))
            assert covered == list(range(n))
            sizes = [shard_range(n, r, world)[1] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch
    n, T, V = 37, 16, 50257
    start, size = shard_range(n, rank, world)
    mine = synth.prompt_ids(V, n, T, seed=105)[start:start + size]
    # every rank's shard, gathered only to check it (bench.py gathers nothing but time)
    sizes = [shard_range(n, r, world)[1] for r in range(world)]
    buf = torch.zeros((max(sizes), T), dtype=torch.int32)
    buf[:size] = torch.from_numpy(mine)
    out = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(out, buf)
    t = torch.tensor([float(rank + 1) * 10.0], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        q.put((np.concatenate([o[:s].numpy() for o, s in zip(out, sizes)]), float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_shards_cover_the_batch():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(got, synth.prompt_ids(50257, 37, 16, seed=105))
    assert tmax == 20.0
