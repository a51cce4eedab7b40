"""Pins the CPU oracle (oracle/murmurate.py) to the reference implementation.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py from
the reference's own reference.py functions; here the oracle restatement must
reproduce them on the CPU: indices exactly, floats to fp32 round-off.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from oracle import murmurate as om

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: (torch.from_numpy(z[k]) if z[k].dtype.kind != "U" else str(z[k])) for k in z.files}


@pytest.mark.parametrize("name", ["config1", "weights_grad", "causal_small", "fp16_inputs",
                                  "bf16_causal"])
def test_oracle_matches_reference_fixture(name):
    f = load(name)
    rounds = int(f["meta_rounds"])
    causal = bool(int(f["meta_causal"]))
    q = f["q"].clone().requires_grad_(True)
    sk = f["slots_k"].clone().requires_grad_(True)
    sv = f["slots_v"].clone().requires_grad_(True)
    out, idx, w = oracle.slot_murmurate(q, sk, sv, rounds=rounds, causal=causal)
    assert torch.equal(idx, f["idx"].long())
    torch.testing.assert_close(out, f["out"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(w, f["w"], atol=1e-6, rtol=1e-5)
    loss = (out * f["grad_out"]).sum()
    if "grad_w" in f:
        loss = loss + (w * f["grad_w"]).sum()
    loss.backward()
    torch.testing.assert_close(q.grad, f["grad_q"], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(sk.grad, f["grad_sk"], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(sv.grad, f["grad_sv"], atol=1e-5, rtol=1e-4)


def test_oracle_matches_reference_round_loop():
    """The north-star composition equals the reference's own slot_murmurate_reference
    (reference.py:138-191) when x = 0 and q_proj = k_proj = v_proj."""
    f = load("reference_loop")
    H = int(f["meta_heads"])
    qp = f["q_proj"]
    B, N, Dm = qp.shape
    q = qp.view(B, N, H, Dm // H).permute(0, 2, 1, 3)
    sk = f["slot_k_emb"].unsqueeze(0).expand(B, -1, -1, -1)
    sv = f["slot_v_emb"].unsqueeze(0).expand(B, -1, -1, -1)
    out, _, _ = oracle.slot_murmurate(q, sk, sv, rounds=int(f["meta_rounds"]))
    torch.testing.assert_close(out.permute(0, 2, 1, 3).reshape(B, N, Dm), f["out"],
                               atol=1e-5, rtol=1e-5)


def test_oracle_phases_match_reference():
    f = load("phases")
    nk, nv = oracle.slot_update(f["tk"], f["tv"], f["slots_k"], f["slots_v"], f["idx"].long(),
                                f["w"], float(f["meta_alpha"]))
    torch.testing.assert_close(nk, f["upd_k"], atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(nv, f["upd_v"], atol=1e-6, rtol=1e-6)
    dk, dv = oracle.slot_diffusion(f["slots_k"], f["slots_v"], float(f["meta_gamma"]))
    torch.testing.assert_close(dk, f["diff_k"], atol=0, rtol=0)
    torch.testing.assert_close(dv, f["diff_v"], atol=0, rtol=0)


@pytest.mark.parametrize("causal", [False, True])
def test_explicit_backward_matches_autograd(causal):
    """The hand-derived backward (the math the CUDA kernels implement) equals
    autograd through the reference composition."""
    g = torch.Generator().manual_seed(11)
    B, H, N, D, M, R = 1, 2, 40, 16, 24, 3
    q = torch.randn(B, H, N, D, generator=g).requires_grad_(True)
    sk = torch.randn(B, H, M, D, generator=g).requires_grad_(True)
    sv = (torch.randn(B, H, M, D, generator=g) * 0.1).requires_grad_(True)
    go = torch.randn(B, H, N, D, generator=g)
    gw = torch.randn(B, H, N, 7, generator=g)
    out, idx, w = oracle.slot_murmurate(q, sk, sv, rounds=R, causal=causal)
    ((out * go).sum() + (w * gw).sum()).backward()
    dq, dk, dv = oracle.slot_murmurate_backward_explicit(q.detach(), sk.detach(), sv.detach(), go, gw,
                                                         rounds=R, causal=causal)
    torch.testing.assert_close(dq, q.grad, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(dk, sk.grad, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(dv, sv.grad, atol=1e-5, rtol=1e-5)


def test_tie_rule_lowest_index():
    s = torch.full((1, 1, 1, 10), float("-inf"))
    s[..., 4] = 1.0
    idx = om.topk_indices(s)
    assert idx.flatten().tolist() == [4, 0, 1, 2, 3, 5, 6]


def test_topk_must_be_seven():
    q = torch.randn(1, 1, 8, 16)
    s = torch.randn(1, 1, 16, 16)
    with pytest.raises(ValueError):
        oracle.slot_murmurate(q, s, s, top_k=5)


def test_row_gap_flags_near_ties():
    t = torch.tensor([[5.0, 4.0, 3.0, 2.0, 1.0, 0.5, 0.25, 0.1],
                      [5.0, 4.0, 3.0, 2.0, 1.0, 0.5, 0.25, 0.25 - 1e-7]])
    assert om.row_gap_ok(t).tolist() == [True, False]


def surface_inputs():
    """The ``surface`` fixture's inputs and its position-bias function."""
    import sys
    sys.path.insert(0, GOLDEN)
    from make_golden import surface_bias_fn
    f = load("surface")
    names = ("x", "q_proj", "k_proj", "v_proj", "slot_k_emb", "slot_v_emb")
    return f, names, surface_bias_fn(f["slot_k_emb"].shape[1])


def test_oracle_full_surface_matches_reference():
    """The full op (reference.py:138-191): residual x, separate token keys and values, a
    mask, a position bias from x, dynamic M — output and every input gradient."""
    f, names, bias_fn = surface_inputs()
    leaves = [f[n].clone().requires_grad_(True) for n in names]
    out = om.slot_murmurate_full(*leaves, num_heads=int(f["meta_heads"]), rounds=int(f["meta_rounds"]),
                                 mask=f["mask"].to(torch.uint8), position_bias_fn=bias_fn,
                                 use_dynamic_m=bool(int(f["meta_use_dynamic_m"])))
    torch.testing.assert_close(out, f["out"], atol=1e-5, rtol=1e-5)
    (out * f["grad_out"]).sum().backward()
    for n, t in zip(names, leaves):
        torch.testing.assert_close(t.grad, f["grad_" + n], atol=1e-5, rtol=1e-4, msg=n)


def test_forced_oracle_with_its_own_picks_is_the_oracle():
    """oracle.slot_murmurate_forced given the oracle's own per-round picks reproduces
    oracle.slot_murmurate exactly (outputs, weights, gradients) on a reference fixture's inputs,
    and reports those picks as its own top-7."""
    f = load("causal_small")
    rounds, causal = int(f["meta_rounds"]), bool(int(f["meta_causal"]))
    q, sk, sv, go = (f[k].float() for k in ("q", "slots_k", "slots_v", "grad_out"))
    tr = om.slot_murmurate_trace(q, sk, sv, rounds, causal)
    a = [t.clone().requires_grad_(True) for t in (q, sk, sv)]
    b = [t.clone().requires_grad_(True) for t in (q, sk, sv)]
    o1, i1, w1 = om.slot_murmurate(*a, rounds=rounds, causal=causal)
    o2, w2, info = om.slot_murmurate_forced(*b, tr["idx"], causal=causal)
    assert torch.equal(o1, o2) and torch.equal(w1, w2)
    assert all(torch.equal(x, y) for x, y in zip(info["own_idx"], tr["idx"]))
    (o1 * go).sum().backward()
    (o2 * go).sum().backward()
    for x, y in zip(a, b):
        assert torch.equal(x.grad, y.grad)
