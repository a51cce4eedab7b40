"""Multi-process host logic on CPU ranks (gloo, world size 2): (batch, head)
sharding round trips, the data-parallel gradient all-reduce, and a rank that
leaves between data-parallel steps (the survivor's next collective must end
with an error within the process group's timeout)."""
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


class _Toy(torch.nn.Module):
    """Two bias-free Linear layers and a free parameter, like the layer's projections and
    slot embeddings."""

    def __init__(self):
        super().__init__()
        torch.manual_seed(1)
        self.a = torch.nn.Linear(6, 5, bias=False)
        self.b = torch.nn.Linear(5, 4, bias=False)
        self.emb = torch.nn.Parameter(torch.randn(4))

    def forward(self, x):
        return self.b(torch.tanh(self.a(x))) + self.emb


def _train_worker(rank, world, port, results):
    """Two ranks take one data-parallel step on their own batches; the parameters must
    match one step on the union of the batches (equal batch sizes: the mean of the ranks'
    gradients is the gradient of the global mean loss)."""
    from murmurative_attention_b200.training import GradientAverager, dp_train_step
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        xs = [torch.randn(3, 6, generator=g) for _ in range(world)]
        model = _Toy()
        opt = torch.optim.SGD(model.parameters(), lr=0.1)
        avg = GradientAverager(model.parameters())
        dp_train_step(model, xs[rank], opt, avg)
        avg.remove()
        ref = _Toy()
        ref_opt = torch.optim.SGD(ref.parameters(), lr=0.1)
        ref(torch.cat(xs)).square().mean().backward()
        ref_opt.step()
        results[rank] = all(torch.allclose(p, q, atol=1e-6) for p, q in zip(model.parameters(), ref.parameters()))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_dp_train_step_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_train_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(results) == {0: True, 1: True}


def _leaver_worker(rank, world, port, results):
    """Both ranks take one data-parallel step; then rank 1 leaves (between steps, with no
    collective in flight) and rank 0's next step must end with an error from its gradient
    all-reduce within the process group's short timeout, not hang."""
    import datetime
    import time
    from murmurative_attention_b200.training import GradientAverager, dp_train_step
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    model = _Toy()
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    avg = GradientAverager(model.parameters())
    x = torch.randn(3, 6, generator=torch.Generator().manual_seed(rank))
    dp_train_step(model, x, opt, avg)
    dist.barrier()
    if rank == 1:
        results[rank] = "left"
        os._exit(0)  # leaves without a goodbye
    time.sleep(0.5)
    t0 = time.monotonic()
    try:
        dp_train_step(model, x, opt, avg)
        results[rank] = ("completed", time.monotonic() - t0)
    except Exception as e:  # noqa: BLE001 — the collective's error, whatever its class
        results[rank] = ("error", time.monotonic() - t0, type(e).__name__)
    os._exit(0)  # the group cannot be torn down cleanly without its peer


def test_gloo_rank_leaving_between_steps_ends_survivors_next_step_with_an_error():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results[1] == "left"
    kind, seconds = results[0][0], results[0][1]
    assert kind == "error", results[0]
    assert seconds < 30, results[0]
