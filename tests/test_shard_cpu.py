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


def _failing_worker(rank, world, port, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                           timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(3)  # this rank fails after joining, before the weight broadcast
    from computeengine_b200.shard import broadcast_from_rank0_checked
    import time
    t0 = time.time()
    ok, msg, sent = broadcast_from_rank0_checked([torch.ones(1 << 16)])
    q.put((ok, msg, sent, time.time() - t0))
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def test_rank_failure_before_broadcast_returns_status():
    """Rank 1 exits after joining the group; rank 0's weight broadcast ends
    with an error status (peer gone or the group's 10 s timeout) instead of
    hanging.  Host-side failure injection only: no GPU is involved."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 150
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    ok, msg, sent, dt = q.get(timeout=5)
    assert not ok and sent == 0 and msg
    assert dt < 60
    assert procs[0].exitcode == 0


def test_parse_cpulist():
    from computeengine_b200.shard import parse_cpulist
    assert parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert parse_cpulist("5") == [5]
    assert parse_cpulist("") == []


def test_pci_local_cpus_reads_sysfs(tmp_path):
    from computeengine_b200.shard import pci_local_cpus
    dev = tmp_path / "0000:1b:00.0"
    dev.mkdir()
    (dev / "local_cpulist").write_text("0-1,4\n")
    assert pci_local_cpus(0, 0x1B, 0, sysfs=str(tmp_path)) == [0, 1, 4]
    assert pci_local_cpus(0, 0x2B, 0, sysfs=str(tmp_path)) is None  # no such device


def test_bind_to_pci_local_cpus_intersects_and_restores(tmp_path):
    import os
    from computeengine_b200.shard import bind_to_pci_local_cpus
    if not hasattr(os, "sched_getaffinity"):
        pytest.skip("no CPU affinity on this platform")
    before = set(os.sched_getaffinity(0))
    one = min(before)
    dev = tmp_path / "0000:00:05.0"
    dev.mkdir()
    # a local set that overlaps the current affinity in one CPU, plus CPUs it lacks
    (dev / "local_cpulist").write_text(f"{one},{max(before) + 1}-{max(before) + 4}\n")
    prev = bind_to_pci_local_cpus(0, 0, 5, sysfs=str(tmp_path))
    try:
        if len(before) == 1:
            assert prev is None  # already bound to that CPU: nothing to change
        else:
            assert prev == before and set(os.sched_getaffinity(0)) == {one}
    finally:
        os.sched_setaffinity(0, before)
    # no overlap at all: affinity left alone
    (dev / "local_cpulist").write_text(f"{max(before) + 10}\n")
    assert bind_to_pci_local_cpus(0, 0, 5, sysfs=str(tmp_path)) is None
    assert set(os.sched_getaffinity(0)) == before
