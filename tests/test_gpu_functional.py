"""The reference's full op surface (murmurative_attention_b200.functional, the per-phase
C ABI) against the oracle on the same inputs: every phase forward and backward (autograd
through the oracle's restatement of reference.py), and the 6-argument round loop against
the reference's own outputs and gradients (tests/golden/surface.npz).

Tolerances: fp32 1e-4 (slot sums are taken in token order, the reference scatter-adds in
pick order); fp16/bf16 atol 2e-3 / 3e-3, rtol 1e-2. Indices: exact on every row whose
top-8 scores are separated by more than 1e-5 of the row's largest (oracle.row_gap_ok);
outputs and gradients are compared on the kernel's own indices.
"""
import os
import sys

import pytest
import torch

from murmurative_attention_b200 import functional as F
from oracle import murmurate as om

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = {torch.float32: dict(atol=1e-4, rtol=1e-4), torch.float16: dict(atol=2e-3, rtol=1e-2),
       torch.bfloat16: dict(atol=3e-3, rtol=1e-2)}


def close(a, b, dt, scale=1.0):
    t = TOL[dt]
    torch.testing.assert_close(a.detach().float().cpu(), b.detach().float().cpu(), atol=t["atol"] * scale,
                               rtol=t["rtol"])


def rnd(g, *shape, std=1.0, dt=torch.float32):
    return (torch.randn(*shape, generator=g) * std).to(dt)


@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", ["plain", "mask_bias", "causal_dyn", "d32_m100"])
def test_select_attend_forward_backward(dt, case):
    g = torch.Generator().manual_seed(11)
    B, H, N, M, D = 2, 3, 70, 64, 64
    if case == "d32_m100":
        M, D = 100, 32
    q = rnd(g, B, H, N, D, dt=dt)
    sk = rnd(g, B, H, M, D, dt=dt)
    sv = rnd(g, B, H, M, D, std=0.5, dt=dt)
    mask = bias = None
    causal, em = False, 0
    if case == "mask_bias":
        mask = (torch.rand(B, 1, N, M, generator=g) > 0.2).to(torch.uint8)
        mask[..., :8] = 1                                  # every row keeps >= 8 selectable slots
        bias = rnd(g, 1, H, N, M, std=0.5, dt=dt)
    if case == "causal_dyn":
        causal, em = True, 48
    go = rnd(g, B, H, N, D, dt=dt)
    gw = rnd(g, B, H, N, 7)
    # device
    qd, skd, svd = (t.cuda().requires_grad_(True) for t in (q, sk, sv))
    out, w, idx = F.slot_select_attend(qd, skd, svd, mask=mask, causal=causal,
                                       position_bias=bias.cuda() if bias is not None else None, effective_M=em)
    ((out.float() * go.cuda().float()).sum() + (w * gw.cuda()).sum()).backward()
    # oracle in fp32 on the same (rounded) inputs
    qo, sko, svo = (t.float().clone().requires_grad_(True) for t in (q, sk, sv))
    scores = om.slot_scores(qo.detach(), sko.detach(), mask=mask, causal=causal,
                            position_bias=bias.float() if bias is not None else None,
                            effective_M=em if em else None)
    ridx = om.topk_indices(scores)
    ok = om.row_gap_ok(torch.sort(scores, dim=-1, descending=True).values[..., :8])
    assert float(ok.float().mean()) > 0.95
    assert torch.equal(idx.cpu()[ok], ridx[ok])
    # attend and backward on the kernel's own indices (the selection is checked above)
    ro, rw = om.slot_attend(qo, sko, svo, idx.cpu())
    ((ro * go.float()).sum() + (rw * gw).sum()).backward()
    close(out, ro, dt)
    close(w, rw, dt)
    s = 4.0 if dt != torch.float32 else 1.0
    close(qd.grad, qo.grad, dt, s)
    close(skd.grad, sko.grad, dt, s)
    close(svd.grad, svo.grad, dt, s)


@pytest.mark.parametrize("M", [256, 300])
def test_select_ties_take_the_lowest_slot(M):
    """Equal scores rank by ascending slot (the oracle's stable sort): every key row appears
    four times, at slots r, r+64, r+128, r+192 (the same lane of the selecting warp and other
    lanes), so each row's top 7 is a four-way tie and three of the next one. M = 256 takes the
    four-token select kernel, M = 300 the one-token kernel."""
    g = torch.Generator().manual_seed(14)
    B, H, N, D = 1, 2, 41, 64
    base = rnd(g, B, H, 64, D)
    sk = torch.cat([base] * (M // 64) + [base[:, :, : M % 64]], dim=2)
    q, sv = rnd(g, B, H, N, D), rnd(g, B, H, M, D)
    out, w, idx = F.slot_select_attend(q.cuda(), sk.cuda(), sv.cuda())
    scores = om.slot_scores(q, sk)
    distinct = torch.sort(scores[..., :64], dim=-1, descending=True).values[..., :3]
    ok = om.row_gap_ok(distinct)
    assert float(ok.float().mean()) > 0.9
    assert torch.equal(idx.cpu()[ok], om.topk_indices(scores)[ok])
    ro, rw = om.slot_attend(q, sk, sv, idx.cpu())
    close(out, ro, torch.float32)
    close(w, rw, torch.float32)


def test_slot_attend_given_indices_clamps():
    g = torch.Generator().manual_seed(12)
    B, H, N, M, D = 1, 2, 33, 40, 16
    q, sk, sv = rnd(g, B, H, N, D), rnd(g, B, H, M, D), rnd(g, B, H, M, D)
    idx = torch.randint(-3, M + 3, (B, H, N, 7), generator=g)
    out, w = F.slot_attend(q.cuda(), sk.cuda(), sv.cuda(), idx.cuda())
    ro, rw = om.slot_attend(q, sk, sv, idx)
    close(out, ro, torch.float32)
    close(w, rw, torch.float32)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_slot_update_forward_backward_with_repeated_indices(dt):
    g = torch.Generator().manual_seed(13)
    B, H, N, M, D = 2, 2, 96, 48, 64
    tk, tv = rnd(g, B, H, N, D, dt=dt), rnd(g, B, H, N, D, dt=dt)
    sk, sv = rnd(g, B, H, M, D, dt=dt), rnd(g, B, H, M, D, dt=dt)
    idx = torch.randint(0, M, (B, H, N, 7), generator=g)      # repeats within a token allowed
    idx[0, 0, 0] = torch.tensor([3, 3, 3, 5, 5, 9, 10])
    w = torch.rand(B, H, N, 7, generator=g)
    w = w / w.sum(-1, keepdim=True)
    gk, gv = rnd(g, B, H, M, D, dt=dt), rnd(g, B, H, M, D, dt=dt)
    dev = [t.cuda().requires_grad_(True) for t in (tk, tv, sk, sv)]
    wd = w.cuda().requires_grad_(True)
    nk, nv = F.slot_update(*dev, idx.cuda(), wd, 0.9)
    ((nk.float() * gk.cuda().float()).sum() + (nv.float() * gv.cuda().float()).sum()).backward()
    ref = [t.float().clone().requires_grad_(True) for t in (tk, tv, sk, sv)]
    wr = w.clone().requires_grad_(True)
    rk, rv = om.slot_update(*ref, idx, wr, 0.9)
    ((rk * gk.float()).sum() + (rv * gv.float()).sum()).backward()
    close(nk, rk, dt)
    close(nv, rv, dt)
    s = 4.0 if dt != torch.float32 else 1.0
    for a, b in zip(dev, ref):
        close(a.grad, b.grad, dt, s)
    close(wd.grad, wr.grad, dt, s)


def test_slot_update_and_diffusion_match_reference_fixture():
    import numpy as np
    z = np.load(os.path.join(GOLDEN, "phases.npz"))
    t = {k: torch.from_numpy(z[k]) for k in z.files}
    nk, nv = F.slot_update(t["tk"].cuda(), t["tv"].cuda(), t["slots_k"].cuda(), t["slots_v"].cuda(),
                           t["idx"].long().cuda(), t["w"].cuda(), float(t["meta_alpha"]))
    close(nk, t["upd_k"], torch.float32)
    close(nv, t["upd_v"], torch.float32)
    dk, dv = F.slot_diffusion(t["slots_k"].cuda(), t["slots_v"].cuda(), float(t["meta_gamma"]))
    assert torch.equal(dk.cpu(), t["diff_k"]) and torch.equal(dv.cpu(), t["diff_v"])


def test_slot_diffusion_backward_is_the_transpose():
    g = torch.Generator().manual_seed(14)
    sk, sv = rnd(g, 1, 2, 30, 16), rnd(g, 1, 2, 30, 16)
    gk, gv = rnd(g, 1, 2, 30, 16), rnd(g, 1, 2, 30, 16)
    a, b = sk.cuda().requires_grad_(True), sv.cuda().requires_grad_(True)
    ok, ov = F.slot_diffusion(a, b, 0.15)
    ((ok * gk.cuda()).sum() + (ov * gv.cuda()).sum()).backward()
    ra, rb = sk.clone().requires_grad_(True), sv.clone().requires_grad_(True)
    rk, rv = om.slot_diffusion(ra, rb, 0.15)
    ((rk * gk).sum() + (rv * gv).sum()).backward()
    close(a.grad, ra.grad, torch.float32)
    close(b.grad, rb.grad, torch.float32)


def test_full_surface_matches_reference_fixture():
    """ops.slot_murmurate's 6-argument loop: residual x, separate q/k/v projections, a
    mask, a position bias recomputed from x, dynamic M — output and all six gradients."""
    import numpy as np
    sys.path.insert(0, GOLDEN)
    from make_golden import surface_bias_fn
    z = np.load(os.path.join(GOLDEN, "surface.npz"))
    f = {k: torch.from_numpy(z[k]) for k in z.files}
    names = ("x", "q_proj", "k_proj", "v_proj", "slot_k_emb", "slot_v_emb")
    leaves = [f[n].cuda().requires_grad_(True) for n in names]
    M = f["slot_k_emb"].shape[1]
    out = F.slot_murmurate(*leaves, num_heads=int(f["meta_heads"]), rounds=int(f["meta_rounds"]),
                           mask=f["mask"].to(torch.uint8).cuda(), position_bias_fn=surface_bias_fn(M),
                           use_dynamic_m=True)
    close(out, f["out"], torch.float32)
    (out * f["grad_out"].cuda()).sum().backward()
    for n, t in zip(names, leaves):
        close(t.grad, f["grad_" + n], torch.float32, 2.0)


def test_full_surface_bf16_against_oracle():
    g = torch.Generator().manual_seed(15)
    B, N, H, Dh, M = 2, 128, 4, 32, 64
    dt = torch.bfloat16
    ins = [rnd(g, B, N, H * Dh, dt=dt) for _ in range(4)] + [rnd(g, H, M, Dh, dt=dt), rnd(g, H, M, Dh, std=0.5, dt=dt)]
    out = F.slot_murmurate(*[t.cuda() for t in ins], num_heads=H, rounds=3, use_dynamic_m=False, causal=True)
    ref = om.slot_murmurate_full(*[t.float() for t in ins], num_heads=H, rounds=3, causal=True)
    rel = ((out.float().cpu() - ref).norm() / ref.norm()).item()
    assert rel < 2e-2


def test_errors_follow_the_reference():
    q = torch.zeros(1, 1, 8, 16, dtype=torch.int32, device="cuda")
    with pytest.raises(TypeError):
        F.slot_select_attend(q, q, q)
    x = torch.zeros(1, 1, 8, 16)
    with pytest.raises(RuntimeError):
        F.slot_select_attend(x, torch.zeros(1, 1, 16, 16), torch.zeros(1, 1, 16, 16))
