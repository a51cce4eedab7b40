"""Forward + backward over host buffers (``slot_murmurate_host_step``, the C ABI's
``murm_slot_murmurate_host_step``): the pipelined copy-in / compute / copy-out path gives the
same results as the device op run on the same (batch, head) groups, bit for bit, and matches
the device op on the whole problem within the fused path's tolerances.
"""
import pytest
import torch

from murmurative_attention_b200 import slot_murmurate, slot_murmurate_host_step

pytestmark = pytest.mark.gpu


def _inputs(B, H, N, M, D, dt, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g).to(dt).pin_memory()
    sk = torch.randn(B, H, M, D, generator=g).to(dt).pin_memory()
    sv = (torch.randn(B, H, M, D, generator=g) * 0.5).to(dt).pin_memory()
    go = torch.randn(B, H, N, D, generator=g).to(dt).pin_memory()
    return q, sk, sv, go


def _device_step(q, sk, sv, go, causal):
    qd, skd, svd = (t.cuda().requires_grad_(True) for t in (q, sk, sv))
    out, idx, w = slot_murmurate(qd, skd, svd, rounds=3, causal=causal)
    out.backward(go.cuda())
    return [t.detach().cpu() for t in (out, idx, w, qd.grad, skd.grad, svd.grad)]


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("causal", [False, True])
def test_groups_match_the_device_op_per_group(dt, causal):
    B, H, N, M, D = 2, 3, 300, 64, 64
    q, sk, sv, go = _inputs(B, H, N, M, D, dt, 41)
    res = slot_murmurate_host_step(q, sk, sv, go, rounds=3, causal=causal, groups=3)
    # groups of 2 (b,h) pairs over the flattened B*H axis: run the device op on the same groups
    flat = lambda t: t.reshape(1, B * H, *t.shape[2:])
    ref = [[] for _ in range(6)]
    for p0 in range(0, B * H, 2):
        part = _device_step(*(flat(t)[:, p0:p0 + 2].contiguous() for t in (q, sk, sv, go)), causal)
        for acc, t in zip(ref, part):
            acc.append(t)
    for got, pieces in zip(res, ref):
        want = torch.cat(pieces, dim=1).reshape(got.shape)
        assert torch.equal(got, want)


def test_one_group_equals_the_device_op_and_many_groups_agree():
    B, H, N, M, D = 1, 8, 1024, 256, 64
    q, sk, sv, go = _inputs(B, H, N, M, D, torch.float16, 42)
    one = slot_murmurate_host_step(q, sk, sv, go, groups=1)
    dev = _device_step(q, sk, sv, go, False)
    for a, b in zip(one, dev):
        assert torch.equal(a, b)
    many = slot_murmurate_host_step(q, sk, sv, go, groups=8)
    # other groupings change only the fp32 order of the chunk partial sums
    assert (many[1] == one[1]).float().mean() > 0.999
    for a, b in zip((many[0], many[3], many[4], many[5]), (one[0], one[3], one[4], one[5])):
        torch.testing.assert_close(a.float(), b.float(), atol=2e-3, rtol=1e-2)


def test_outputs_are_reused_and_errors_follow_the_reference():
    q, sk, sv, go = _inputs(1, 2, 64, 32, 32, torch.float32, 43)
    outs = tuple(torch.empty_like(t) for t in (q,)) + (
        torch.empty(1, 2, 64, 7, dtype=torch.int64), torch.empty(1, 2, 64, 7), torch.empty_like(q),
        torch.empty_like(sk), torch.empty_like(sv))
    res = slot_murmurate_host_step(q, sk, sv, go, outputs=outs)
    assert all(a is b for a, b in zip(res, outs))
    with pytest.raises(TypeError):
        slot_murmurate_host_step(q.int(), sk, sv, go)
    with pytest.raises(RuntimeError):
        slot_murmurate_host_step(q.cuda(), sk, sv, go)
