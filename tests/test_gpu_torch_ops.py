"""torch.ops.murmurative_attention on the GPU: the reference's seven operators
(torch-ext/torch_binding.cpp:6-43) as callers reach them through the dispatcher
(src/murmurative/ops.py:30-38), and the north-star operator with autograd. Each matches the
library's own Python entry points bitwise (the same kernels run), and torch.compile(fullgraph=True)
traces the MurmurativeAttention layer through the registered operator."""
import pytest
import torch

import murmurative_attention_b200 as mab
from murmurative_attention_b200 import functional as F

pytestmark = pytest.mark.gpu
NS = torch.ops.murmurative_attention


def _inputs(seed, B=2, H=3, N=200, M=64, D=64, dt=torch.float16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, H, N, D, device="cuda", generator=g).to(dt)
    k = torch.randn(B, H, N, D, device="cuda", generator=g).to(dt)
    v = torch.randn(B, H, N, D, device="cuda", generator=g).to(dt)
    sk = torch.randn(B, H, M, D, device="cuda", generator=g).to(dt)
    sv = (torch.randn(B, H, M, D, device="cuda", generator=g) * 0.3).to(dt)
    return q, k, v, sk, sv


def _eq(a, b):
    assert len(a) == len(b)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("dt", [torch.float16, torch.float32])
def test_select_attend_and_backward(dt):
    q, _, _, sk, sv = _inputs(1, dt=dt)
    mask = (torch.rand(q.shape[2], sk.shape[2], device="cuda") > 0.2).to(torch.uint8)
    out = NS.slot_select_attend(q, sk, sv, mask, True, None, None, 48)
    ref = F.slot_select_attend(q, sk, sv, mask, True, None, None, 48)
    _eq(out, ref)
    o, w, idx = out
    go = torch.randn_like(o)
    gw = torch.randn_like(w)
    grads = NS.slot_select_attend_backward(go, gw, q, sk, sv, idx, w, None)
    qa, ska, sva = (t.clone().requires_grad_(True) for t in (q, sk, sv))
    o2, w2, _ = F.slot_select_attend(qa, ska, sva, mask, True, None, None, 48)
    ((o2.float() * go.float()).sum() + (w2 * gw).sum()).backward()
    _eq(grads, (qa.grad, ska.grad, sva.grad))


def test_update_diffusion_in_place_and_backward():
    q, k, v, sk, sv = _inputs(2)
    _, w, idx = F.slot_select_attend(q, sk, sv)
    nk, nv = F.slot_update(k, v, sk, sv, idx, w, 0.9)
    a, b = sk.clone(), sv.clone()
    NS.slot_update(a, b, k, v, idx, w, 0.9)
    _eq((a, b), (nk, nv))
    dk, dv = F.slot_diffusion(nk, nv, 0.15)
    NS.slot_diffusion(a, b, 0.15)
    _eq((a, b), (dk, dv))
    c, d = sk.clone(), sv.clone()
    NS.slot_update_diffuse(c, d, k, v, idx, w, 0.9, 0.15)
    _eq((c, d), (dk, dv))
    gnk, gnv = torch.randn_like(nk), torch.randn_like(nv)
    ka, va, ska, sva, wa = (t.clone().requires_grad_(True) for t in (k, v, sk, sv, w))
    ok, ov = F.slot_update(ka, va, ska, sva, idx, wa, 0.9)
    ((ok.float() * gnk.float()).sum() + (ov.float() * gnv.float()).sum()).backward()
    _eq(NS.slot_update_backward(gnk, gnv, k, v, idx, w, 0.9), (ka.grad, va.grad, ska.grad, sva.grad, wa.grad))
    xk, xv = (t.clone().requires_grad_(True) for t in (nk, nv))
    yk, yv = F.slot_diffusion(xk, xv, 0.15)
    ((yk.float() * gnk.float()).sum() + (yv.float() * gnv.float()).sum()).backward()
    _eq(NS.slot_diffusion_backward(gnk, gnv, 0.15), (xk.grad, xv.grad))


@pytest.mark.parametrize("dt,causal", [(torch.float16, False), (torch.bfloat16, True)])
def test_north_star_operator_with_autograd(dt, causal):
    q, _, _, sk, sv = _inputs(3, N=700, M=256, dt=dt)
    go = torch.randn_like(q)
    gw = torch.randn(*q.shape[:3], 7, device="cuda")
    res = []
    for fn in (mab.slot_murmurate, NS.slot_murmurate):
        qa, ska, sva = (t.clone().requires_grad_(True) for t in (q, sk, sv))
        out, idx, w = fn(qa, ska, sva, 3, 7, causal)
        ((out.float() * go.float()).sum() + (w * gw).sum()).backward()
        res.append((out, idx, w, qa.grad, ska.grad, sva.grad))
    _eq(res[0], res[1])


def test_layer_compiles_fullgraph():
    torch.manual_seed(0)
    layer = mab.MurmurativeAttention(256, 4, 64, rounds=3).cuda().to(torch.bfloat16)
    x = torch.randn(2, 300, 256, device="cuda", dtype=torch.bfloat16)
    eager = layer(x)
    eager.float().square().mean().backward()
    g_eager = [p.grad.clone() for p in layer.parameters()]
    layer.zero_grad(set_to_none=True)
    compiled = torch.compile(layer, fullgraph=True)
    out = compiled(x)
    out.float().square().mean().backward()
    torch.testing.assert_close(out.float(), eager.float(), atol=2e-3, rtol=1e-2)
    for a, b in zip([p.grad for p in layer.parameters()], g_eager):
        torch.testing.assert_close(a.float(), b.float(), atol=2e-3, rtol=1e-2)
