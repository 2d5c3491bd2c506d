"""Host logic of the multi-GPU path, on CPU: the longest-processing-time stream sharding and,
with two gloo ranks, the rank-0 decision every rank agrees on and the max-over-ranks stats
gather (the one collective of a bench run)."""
from __future__ import annotations

import importlib
import os
import socket

import numpy as np
import pytest

from conftest import load_package

load_package()
sharding = importlib.import_module("moss_b200.sharding")


def test_lpt_shard_covers_every_stream_once_with_fixed_counts():
    rng = np.random.default_rng(1234)
    lens = [int(x) for x in rng.integers(64, 1025, 8 * 64)]
    shards = sharding.lpt_shard(lens, 8, per_rank=64)
    assert sorted(i for s in shards for i in s) == list(range(len(lens)))
    assert all(len(s) == 64 for s in shards)
    totals = [sum(lens[i] for i in s) for s in shards]
    # LPT with equal counts: the spread is at most the longest stream
    assert max(totals) - min(totals) <= max(lens)
    assert max(totals) / (sum(lens) / 8) < 1.01


def test_lpt_shard_is_deterministic_and_handles_edge_cases():
    assert sharding.lpt_shard([5, 5, 5, 5], 2) == sharding.lpt_shard([5, 5, 5, 5], 2)
    assert sharding.lpt_shard([], 3) == [[], [], []]
    assert sharding.lpt_shard([7], 1) == [[0]]
    with pytest.raises(ValueError):
        sharding.lpt_shard([1, 2, 3], 1, per_rank=2)
    with pytest.raises(ValueError):
        sharding.lpt_shard([1], 0)


def _worker(rank, world, port, lens, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shards = sharding.agree_shards(dist, lens, per_rank=len(lens) // world)
        mine = shards[rank]
        gathered = [None] * world
        dist.all_gather_object(gathered, (rank, shards))
        worst = sharding.max_over_ranks(dist, float(10 * rank + 1))
        out.put((rank, mine, all(g[1] == shards for g in gathered), worst))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_shards_and_gather_the_max():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    lens = [int(x) for x in np.random.default_rng(7).integers(64, 1025, 16)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lens, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = sharding.lpt_shard(lens, 2, per_rank=8)
    for rank, mine, consistent, worst in res:
        assert consistent
        assert mine == expect[rank]
        assert worst == 11.0
