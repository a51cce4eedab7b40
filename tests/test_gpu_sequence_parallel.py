"""Sequence parallelism (murmurative_attention_b200.sequence_parallel) and the slot-sums
phase it is built on.

The two-rank test runs two processes on one GPU over gloo (CUDA tensors; the kernels of
the two processes never wait on each other), each with half the tokens, and compares the
ranks' outputs, indices, weights and gradients with one process over all tokens and with the
oracle. Slot gradients are per-rank partial sums (like data-parallel gradients); their sum
over the ranks must equal the single-process gradient.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from murmurative_attention_b200 import functional as F
from oracle import murmurate as om

pytestmark = pytest.mark.gpu


def test_slot_sums_forward_backward_match_oracle():
    g = torch.Generator().manual_seed(31)
    B, H, N, M, D = 2, 2, 80, 40, 32
    tk, tv = torch.randn(B, H, N, D, generator=g), torch.randn(B, H, N, D, generator=g)
    idx = torch.randint(0, M, (B, H, N, 7), generator=g)
    w = torch.rand(B, H, N, 7, generator=g)
    gk, gv, gw = torch.randn(B, H, M, D, generator=g), torch.randn(B, H, M, D, generator=g), torch.randn(B, H, M, generator=g)
    a, b, wd = tk.cuda().requires_grad_(True), tv.cuda().requires_grad_(True), w.cuda().requires_grad_(True)
    ks, vs, ws = F.slot_sums(a, b, idx.cuda(), wd, M)
    ((ks * gk.cuda()).sum() + (vs * gv.cuda()).sum() + (ws * gw.cuda()).sum()).backward()
    ra, rb, rw = tk.clone().requires_grad_(True), tv.clone().requires_grad_(True), w.clone().requires_grad_(True)
    rk = torch.zeros(B, H, M, D).index_put_((torch.arange(B).view(B, 1, 1, 1), torch.arange(H).view(1, H, 1, 1), idx),
                                            ra.unsqueeze(3) * rw.unsqueeze(-1), accumulate=True)
    rv = torch.zeros(B, H, M, D).index_put_((torch.arange(B).view(B, 1, 1, 1), torch.arange(H).view(1, H, 1, 1), idx),
                                            rb.unsqueeze(3) * rw.unsqueeze(-1), accumulate=True)
    rs = torch.zeros(B, H, M).index_put_((torch.arange(B).view(B, 1, 1, 1), torch.arange(H).view(1, H, 1, 1), idx),
                                         rw, accumulate=True)
    ((rk * gk).sum() + (rv * gv).sum() + (rs * gw).sum()).backward()
    for x, y in ((ks, rk), (vs, rv), (ws, rs), (a.grad, ra.grad), (b.grad, rb.grad), (wd.grad, rw.grad)):
        torch.testing.assert_close(x.detach().cpu(), y.detach(), atol=1e-4, rtol=1e-4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(causal):
    g = torch.Generator().manual_seed(32)
    B, H, N, M, D = 1, 2, 256, 64, 64
    q = torch.randn(B, H, N, D, generator=g)
    sk = torch.randn(B, H, M, D, generator=g)
    sv = torch.randn(B, H, M, D, generator=g) * 0.3
    go = torch.randn(B, H, N, D, generator=g)
    return q, sk, sv, go


def _run(q, sk, sv, go, causal, group=None):
    from murmurative_attention_b200.sequence_parallel import slot_murmurate_sp
    qd, skd, svd = (t.cuda().requires_grad_(True) for t in (q, sk, sv))
    out, idx, w = slot_murmurate_sp(qd, skd, svd, rounds=3, causal=causal, group=group)
    (out * go.cuda()).sum().backward()
    return {k: v.detach().cpu() for k, v in dict(out=out, idx=idx, w=w, gq=qd.grad, gsk=skd.grad, gsv=svd.grad).items()}


def _rank(rank, world, port, causal, results):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, sk, sv, go = _inputs(causal)
        n = q.shape[2] // world
        sl = slice(rank * n, (rank + 1) * n)
        results[rank] = _run(q[:, :, sl].contiguous(), sk, sv, go[:, :, sl].contiguous(), causal)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("causal", [False, True])
def test_two_ranks_match_one(causal):
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, causal, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    # one process, all tokens (no collective at world size 1)
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        full = _run(*_inputs(causal), causal)
    finally:
        dist.destroy_process_group()
    r0, r1 = results[0], results[1]
    cat = lambda k: torch.cat([r0[k], r1[k]], dim=2)
    assert torch.equal(cat("idx"), full["idx"])
    torch.testing.assert_close(cat("out"), full["out"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(cat("w"), full["w"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(cat("gq"), full["gq"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(r0["gsk"] + r1["gsk"], full["gsk"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(r0["gsv"] + r1["gsv"], full["gsv"], atol=1e-4, rtol=1e-4)
    # and the two-rank composition against the oracle (reference.py:177-189, with the slot sums
    # of reference.py:87-103 all-reduced over the token shards): fp32, every row unambiguous here
    q, sk, sv, go = _inputs(causal)
    qf, skf, svf = (t.clone().requires_grad_(True) for t in (q, sk, sv))
    ro, ri, rw = om.slot_murmurate(qf, skf, svf, rounds=3, causal=causal)
    (ro * go).sum().backward()
    ok = om.row_gap_ok(om.slot_murmurate_trace(q, sk, sv, 3, causal)["top8"][-1])
    assert bool(ok.all()), "these seeded inputs have no near-tie rows"
    assert torch.equal(cat("idx"), ri)
    torch.testing.assert_close(cat("out"), ro.detach(), atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(cat("w"), rw.detach(), atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(cat("gq"), qf.grad, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(r0["gsk"] + r1["gsk"], skf.grad, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(r0["gsv"] + r1["gsv"], svf.grad, atol=1e-4, rtol=1e-4)
