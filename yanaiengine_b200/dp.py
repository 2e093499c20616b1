"""Data-parallel sharding of independent sequences across GPUs (one process per GPU).

Every GPU holds a full target + draft replica, its own KV pool and its own
block allocator; sequences never interact, so there is no collective on the
data path.  The host splits a global request list across ranks with a
count-capped longest-first greedy (each rank gets ceil(n / world) or fewer
sequences; a sequence goes to the rank with the least total context so far,
KV bytes being proportional to context), and the job reduces two scalars at
the end: the slowest rank's device time and the total emitted tokens.
"""
from __future__ import annotations

import numpy as np


def partition(lengths, world: int) -> list[list[int]]:
    """Indices of `lengths` per rank: longest first onto the least-loaded rank
    that still has room (at most ceil(n / world) sequences per rank); ties go
    to the lower rank.  Deterministic, so every rank computes the same split."""
    lengths = np.asarray(lengths, dtype=np.int64)
    n = len(lengths)
    if world <= 0:
        raise ValueError("world must be positive")
    cap = -(-n // world)
    order = sorted(range(n), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min((r for r in range(world) if len(out[r]) < cap), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(x) for x in out]


def global_lengths(per_rank: int, world: int, seed: int = 7, lo: int = 512, hi: int = 2048) -> np.ndarray:
    """Context lengths U[lo, hi] of the whole job's per_rank x world sequences."""
    return np.random.default_rng(seed).integers(lo, hi + 1, per_rank * world)


def all_max(world: int, x: float, device: str = "cuda") -> float:
    """Maximum of x over the process group (x itself when world == 1)."""
    return _reduce(world, x, "max", device)


def all_sum(world: int, x: float, device: str = "cuda") -> float:
    """Sum of x over the process group (x itself when world == 1)."""
    return _reduce(world, x, "sum", device)


def _reduce(world: int, x: float, op: str, device: str) -> float:
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())
