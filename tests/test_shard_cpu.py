"""Multi-GPU host logic on the CPU: batch slices, the one-time weight
broadcast from rank 0 and the max-over-ranks timing reduction, run as two
gloo ranks (the B200 runs use NCCL over NVLink with the same calls)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from computeengine_b200.shard import broadcast_from_rank0, max_over_ranks, shard_batch


def test_shard_batch_covers_exactly():
    for gb, world in ((2048, 8), (2048, 3), (5, 4), (0, 2), (256, 1)):
        seen = []
        for r in range(world):
            first, count = shard_batch(gb, world, r)
            seen.extend(range(first, first + count))
        assert seen == list(range(gb))
    with pytest.raises(ValueError):
        shard_batch(8, 2, 2)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # every rank builds "weights" that differ; rank 0's must win
        ws = [torch.full((64,), float(rank + 1)), torch.arange(10, dtype=torch.int32) * (rank + 1)]
        sent = broadcast_from_rank0(ws)
        ok = bool(torch.all(ws[0] == 1.0)) and bool(torch.all(ws[1] == torch.arange(10, dtype=torch.int32)))
        m = max_over_ranks(3.5 + rank)
        q.put((rank, ok, sent, m))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_broadcast_and_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=5) for _ in range(2))
    for rank, ok, sent, m in res:
        assert ok
        assert sent == 64 * 4 + 10 * 4
        assert m == 4.5
