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

import os
from pathlib import Path
from typing import Iterable, List, Optional, Set, Tuple


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


def broadcast_from_rank0_checked(tensors: Iterable) -> Tuple[bool, str, int]:
    """broadcast_from_rank0 with a failed peer turned into a status instead of
    a hang or an exception: (ok, message, bytes sent).  A rank that dies or
    exits before the broadcast makes the collective end with an error, either
    at once (its connection closed) or at the process group's timeout; the
    surviving ranks report that and can shut down cleanly.  Call
    dist.destroy_process_group() afterwards either way."""
    try:
        return True, "", broadcast_from_rank0(tensors)
    except Exception as e:  # the backends raise RuntimeError subclasses (DistBackendError, ...)
        return False, f"{type(e).__name__}: {e}".strip(), 0


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar (e.g. elapsed milliseconds)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def parse_cpulist(text: str) -> List[int]:
    """CPU ids of a sysfs cpulist such as "0-3,8,10-11"."""
    cpus: List[int] = []
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            lo, hi = part.split("-", 1)
            cpus.extend(range(int(lo), int(hi) + 1))
        else:
            cpus.append(int(part))
    return cpus


def pci_local_cpus(domain: int, bus: int, device: int,
                   sysfs: str = "/sys/bus/pci/devices") -> Optional[List[int]]:
    """CPUs attached to the same NUMA node as a PCI device (function 0), or
    None when sysfs does not say."""
    path = Path(sysfs) / f"{domain:04x}:{bus:02x}:{device:02x}.0" / "local_cpulist"
    try:
        cpus = parse_cpulist(path.read_text())
    except (OSError, ValueError):
        return None
    return cpus or None


def bind_to_pci_local_cpus(domain: int, bus: int, device: int,
                           sysfs: str = "/sys/bus/pci/devices") -> Optional[Set[int]]:
    """Restricts this process to the CPUs local to a GPU's PCI address
    (intersected with its current affinity), so that pinned host buffers it
    allocates afterwards are placed on the GPU's own NUMA node by first touch
    and its copies do not cross the socket link.  Returns the previous
    affinity (for os.sched_setaffinity to restore), or None when nothing was
    changed (no sysfs entry, no overlap, or no affinity support)."""
    if not hasattr(os, "sched_getaffinity"):
        return None
    local = pci_local_cpus(domain, bus, device, sysfs)
    if local is None:
        return None
    prev = set(os.sched_getaffinity(0))
    want = prev & set(local)
    if not want or want == prev:
        return None
    os.sched_setaffinity(0, want)
    return prev
