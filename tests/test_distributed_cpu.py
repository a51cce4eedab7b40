"""Multi-process host logic on CPU ranks (gloo, world size 2): (batch, head)
sharding round trips and the data-parallel gradient all-reduce."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from murmurative_attention_b200 import distributed as md


def test_pair_range_covers_all_pairs_once():
    for total in (1, 7, 16, 128, 130):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s, e = md.pair_range(total, world, r)
                seen.extend(range(s, e))
            assert seen == list(range(total))
    with pytest.raises(ValueError):
        md.pair_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # sharding round trip
        g = torch.Generator().manual_seed(0)
        x = torch.randn(3, 5, 4, 2, generator=g)
        loc = md.local_pairs(x, world, rank)
        back = md.gather_pairs(loc.clone(), 3, 5)
        ok_shard = torch.equal(back, x)
        # data-parallel all-reduce: each rank's gradient is rank+1 (and a per-rank pattern)
        lin = torch.nn.Linear(4, 3, bias=False)
        emb = torch.nn.Parameter(torch.zeros(2, 5))
        lin.weight.grad = torch.full_like(lin.weight, float(rank + 1))
        emb.grad = torch.arange(10, dtype=torch.float32).view(2, 5) * (rank + 1)
        md.allreduce_gradients([lin.weight, emb])
        mean = sum(range(1, world + 1)) / world
        ok_w = torch.allclose(lin.weight.grad, torch.full_like(lin.weight, mean))
        ok_e = torch.allclose(emb.grad, torch.arange(10, dtype=torch.float32).view(2, 5) * mean)
        results[rank] = bool(ok_shard and ok_w and ok_e)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_shard_and_allreduce():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(results) == {0: True, 1: True}
