"""Sharding planner: CPU tests, including a world_size-2 gloo run in which
each rank plans independently and the ranks check (by all_gather) that their
shards are disjoint, complete and balanced -- the property that lets the
multi-GPU path run without any collective on the data path."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fmha_native_b200 import shard

CONFIGS = {
    "c2": (4, 16, 2048, 2048, False, None),
    "c3": (1, 16, 8192, 8192, True, None),
    "c5a": (1, 2, 40000, 40000, True, None),
    "c5b": (32, 32, 4096, 4096, True, None),
    "varlen": (4, 8, 0, 0, True, [1, 600, 257, 4096]),
    "asym": (2, 4, 300, 1000, True, None),
}


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_partition_complete_disjoint_balanced(name, world):
    b, h, sq, sk, causal, vl = CONFIGS[name]
    blocks = shard.plan_blocks(b, h, sq, sk, causal, vl)
    parts = shard.partition(blocks, world)
    flat = [(x[0], x[1]) for p in parts for x in p]
    assert sorted(flat) == sorted((x[0], x[1]) for x in blocks)
    assert len(set(flat)) == len(flat)
    L = shard.loads(parts)
    if len(blocks) >= 8 * world:
        assert max(L) <= 1.05 * sum(L) / world
    for p in parts:  # head-major, heavy-first within a head
        assert all((p[i][0], -p[i][2]) <= (p[i + 1][0], -p[i + 1][2]) for i in range(len(p) - 1))


def test_block_costs_causal_monotone():
    costs = [shard.block_cost(m, 4096, 4096, True) for m in range(16)]
    assert costs == sorted(costs) and costs[0] < costs[-1]
    assert shard.block_cost(0, 4096, 4096, False) == shard.block_cost(15, 4096, 4096, False)
    # Sq > Sk causal: the top rows see no key at all
    assert shard.block_cost(0, 1024, 256, True) == shard.BLOCK_OVERHEAD


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, h, sq, sk, causal, vl = CONFIGS["c5b"]
        mine = shard.partition(shard.plan_blocks(b, h, sq, sk, causal, vl), world)[rank]
        gathered = [None] * world
        dist.all_gather_object(gathered, [(x[0], x[1], x[2]) for x in mine])
        if rank == 0:
            flat = [(x[0], x[1]) for p in gathered for x in p]
            total = shard.plan_blocks(b, h, sq, sk, causal, vl)
            loads = [sum(x[2] for x in p) for p in gathered]
            results["ok"] = (len(flat) == len(set(flat)) == len(total) and
                             max(loads) <= 1.01 * sum(loads) / world)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_plan_consistently():
    world = 2
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        assert results.get("ok") is True
