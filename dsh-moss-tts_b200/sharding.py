"""Stream-to-GPU sharding for one process per GPU.

Streams (utterances) are independent, so a multi-GPU job shards them across ranks with no
collective on the data path.  KV lengths are ragged, so the shards are balanced by total KV
length with the longest-processing-time rule: streams in decreasing length, each to the
rank with the least total so far among ranks that still have room (a fixed count per rank
keeps the per-GPU batch shape, hence its captured frame graph, the same on every rank).
Rank 0 decides and broadcasts, so every rank acts on the same assignment; the only other
collective is the max over ranks of the device timings at the end (the stats gather).
"""
from __future__ import annotations

from typing import Sequence


def lpt_shard(lengths: Sequence[int], n_ranks: int, per_rank: int | None = None) -> list[list[int]]:
    """Indices of `lengths` per rank.  Ties go to the lower length index / lower rank, so the
    result is deterministic.  per_rank = None: len(lengths) / n_ranks, rounded up."""
    n = len(lengths)
    if n_ranks <= 0:
        raise ValueError("n_ranks must be positive")
    cap = per_rank if per_rank is not None else -(-n // n_ranks)
    if cap * n_ranks < n:
        raise ValueError(f"{n} streams do not fit {n_ranks} ranks of {cap}")
    order = sorted(range(n), key=lambda i: (-int(lengths[i]), i))
    load = [0] * n_ranks
    shards: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        r = min((k for k in range(n_ranks) if len(shards[k]) < cap), key=lambda k: (load[k], k))
        shards[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(s) for s in shards]


def agree_shards(dist, lengths: Sequence[int], per_rank: int | None = None) -> list[list[int]]:
    """lpt_shard decided on rank 0 and broadcast to every rank of the default process group
    (any backend: gloo on CPU, nccl on GPUs).  Without a process group: world size 1."""
    if dist is None or not dist.is_initialized():
        return lpt_shard(lengths, 1, per_rank)
    world = dist.get_world_size()
    box = [lpt_shard(lengths, world, per_rank) if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def max_over_ranks(dist, value: float, device=None) -> float:
    """The stats gather: the largest value over all ranks (device timings are reported as
    the max over ranks).  device = the tensor device the backend needs (cuda for nccl)."""
    if dist is None or not dist.is_initialized():
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
