"""Batch sharding across GPUs (one process per GPU).

The convolution stack shards over images: rank r of N runs its own
contiguous slice of the global batch; weights, biases and requantize
multipliers are sent once from rank 0 (NCCL over NVLink on B200s, gloo in the
CPU tests); there is no per-layer collective.  Timings are reduced as the
maximum over ranks.  The reference has no distributed execution for this
path (DistributedContext::all_reduce returns Unsupported,
src/train/distributed/distributed.h:29-34).
"""
from __future__ import annotations

from typing import Iterable, Tuple


def shard_batch(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """(first image, image count) of this rank's contiguous slice; slices
    cover the batch exactly, sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world or global_batch < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(global_batch, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def input_seed(base_seed: int, rank: int) -> int:
    """Seed of a rank's synthetic input slice."""
    return base_seed + 1000 + rank


def broadcast_from_rank0(tensors: Iterable) -> int:
    """Sends every tensor from rank 0 to all ranks (in place); returns the
    bytes sent.  A no-op without an initialized process group."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return 0
    total = 0
    for t in tensors:
        dist.broadcast(t, src=0)
        total += t.numel() * t.element_size()
    return total


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar (e.g. elapsed milliseconds)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
