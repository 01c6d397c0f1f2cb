"""Sequence sharding across GPUs: one process per GPU, no collective on the hot path.

RWKV-7 sequences are independent and each one's recurrent state lives on a single
GPU, so a multi-GPU job partitions sequences across ranks (weights replicated) and
every rank runs its own decode / prefill steps. ``torch.distributed`` is used only
around the hot path: to agree on timings (max over ranks) and to gather per-rank
results on rank 0.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["shard_range", "shard_by_length", "max_over_ranks", "gather_to_rank0"]


def shard_range(n_items: int, world: int, rank: int) -> range:
    """Contiguous block of ``n_items`` owned by ``rank`` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def shard_by_length(lengths: list[int], world: int) -> list[list[int]]:
    """Greedy longest-first assignment of sequences to ranks balancing total tokens
    (continuous batching with prompts of different lengths). Returns the sequence
    indices of each rank, each list in increasing order."""
    if world <= 0:
        raise ValueError("world must be positive")
    load = [0] * world
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda j: (-lengths[j], j)):
        r = min(range(world), key=lambda q: (load[q], q))
        owned[r].append(i)
        load[r] += lengths[i]
    return [sorted(o) for o in owned]


def max_over_ranks(x: float, device: torch.device | str = "cpu") -> float:
    """Maximum of a per-rank scalar (e.g. a step time); identity without a process group."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(obj):
    """List of every rank's ``obj`` on rank 0 (None elsewhere); ``[obj]`` without a group."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
    dist.gather_object(obj, out, dst=0)
    return out
