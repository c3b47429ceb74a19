"""Sequence sharding for multi-GPU batched decode (no collective on the data
path): the planner's partition, and the same plan reached independently by
every rank of a 2-process gloo group, as bench.py's ranks do."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from minimind_orangepi_b200.sharding import plan_shards, shard_imbalance


def test_plan_is_a_balanced_partition():
    rng = np.random.default_rng(0)
    ctx = [int(x) + 256 for x in rng.integers(16, 2049, size=256)]
    for world in (1, 2, 4, 8):
        shards = plan_shards(ctx, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(256))
        assert shard_imbalance(ctx, shards) < 1.02
        assert all(len(s) >= 256 // world - 8 for s in shards)


def test_plan_edge_cases():
    assert plan_shards([], 2) == [[], []]
    assert plan_shards([5], 3) == [[0], [], []]
    with pytest.raises(ValueError):
        plan_shards([1], 0)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    ctx = [int(x) for x in rng.integers(16, 2049, size=64)]
    mine = plan_shards(ctx, world)[rank]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    load = [float(sum(ctx[i] for i in mine))]
    import torch
    t = torch.tensor(load)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    out[rank] = (gathered, float(t.item()))
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ranks_agree_on_disjoint_shards_gloo():
    world = 2
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    g0, mx0 = res[0]
    g1, mx1 = res[1]
    assert g0 == g1
    assert sorted(g0[0] + g0[1]) == list(range(64)) and not set(g0[0]) & set(g0[1])
    assert mx0 == mx1
