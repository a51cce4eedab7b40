"""Generate golden fixtures for slot_murmurate from the reference implementation.

Run in a container where the reference (beaglabs/murmurative-attention) is
checked out; it is not needed anywhere else:

    python tests/golden/make_golden.py /path/to/reference/src

(or with the path in MURM_REFERENCE_SRC).

It imports the reference's own ``murmurative.reference`` module and composes
its four functions (slot_select_reference, slot_attend_reference,
slot_update_reference, slot_diffusion_reference) into the north-star op
exactly as the reference round loop does (reference.py:177-189) with token
keys = token values = q and a zero residual. Gradients come from autograd
through those reference functions. Every case is seeded; the outputs are
written as small .npz files next to this script.

Tie rule: torch.topk orders equal scores arbitrarily. For the causal case the
only ties are the -inf scores of rows n < 6; those rows take the lowest-index
masked slots (n+1, n+2, ...). The script asserts that on every other row the
reference's own topk indices equal the lowest-index-rule indices, so nothing
else about selection is assumed.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(src: str):
    sys.path.insert(0, src)
    from murmurative import reference as ref  # noqa: E402
    return ref


def _stable_top7(scores: torch.Tensor) -> torch.Tensor:
    return torch.sort(scores, dim=-1, descending=True, stable=True).indices[..., :7]


def _select(ref, q, sk, causal):
    """Reference select; rows whose 8 largest scores contain a tie use the
    lowest-index rule. Asserts the two agree on every other row."""
    idx_ref = ref.slot_select_reference(q, sk, causal=causal)
    scores = torch.einsum("bhnd,bhmd->bhnm", q, sk)
    if causal:
        M, N = sk.shape[2], q.shape[2]
        scores = scores.masked_fill(torch.arange(M).view(1, 1, 1, M) > torch.arange(N).view(1, 1, N, 1),
                                    float("-inf"))
    top8 = torch.sort(scores, dim=-1, descending=True).values[..., :8]
    tied = (top8[..., 1:] == top8[..., :-1]).any(-1)
    idx_rule = _stable_top7(scores)
    assert torch.equal(idx_ref[~tied], idx_rule[~tied]), "reference topk disagrees on an untied row"
    return torch.where(tied.unsqueeze(-1), idx_rule, idx_ref), int(tied.sum())


def compose(ref, q, sk, sv, rounds, causal, alpha=0.9, gamma=0.15, grad_out=None, grad_w=None):
    q = q.detach().float().requires_grad_(True)
    sk0 = sk.detach().float().requires_grad_(True)
    sv0 = sv.detach().float().requires_grad_(True)
    out = torch.zeros_like(q)
    k, v = sk0, sv0
    ties = 0
    idx = w = None
    for _ in range(rounds):
        idx, t = _select(ref, q.detach(), k.detach(), causal)
        ties += t
        o, w = ref.slot_attend_reference(q, k, v, idx)
        out = out + o
        k, v = ref.slot_update_reference(q, q, k, v, idx, w, alpha)
        k, v = ref.slot_diffusion_reference(k, v, gamma)
    res = dict(out=out.detach(), idx=idx, w=w.detach(), tied_rows=np.int64(ties))
    if grad_out is not None:
        loss = (out * grad_out.float()).sum()
        if grad_w is not None:
            loss = loss + (w * grad_w.float()).sum()
        loss.backward()
        res.update(grad_q=q.grad, grad_sk=sk0.grad, grad_sv=sv0.grad)
    return res


def _save(name, inputs, res, meta):
    arrays = {}
    for k, v in {**inputs, **res}.items():
        if isinstance(v, torch.Tensor):
            v = v.detach()
            if v.dtype == torch.int64:
                arrays[k] = v.numpy().astype(np.int16)
            else:
                arrays[k] = v.float().numpy()
        else:
            arrays[k] = np.asarray(v)
    for k, v in meta.items():
        arrays["meta_" + k] = np.asarray(v)
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    print(f"{name}: {os.path.getsize(path) / 1024:.0f} KiB, tied rows {int(res.get('tied_rows', 0))}")


def _randn(g, *shape, std=1.0, dtype=torch.float32):
    return (torch.randn(*shape, generator=g) * std).to(dtype).float()


def main(src):
    ref = _load_reference(src)
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # 1. the README verify shape, fp32, non-causal, fwd + bwd.
    g = torch.Generator().manual_seed(0)
    q = _randn(g, 2, 4, 128, 64)
    sk = _randn(g, 2, 4, 256, 64)
    sv = torch.zeros(2, 4, 256, 64)
    go = _randn(g, 2, 4, 128, 64)
    res = compose(ref, q, sk, sv, 3, False, grad_out=go)
    _save("config1", dict(q=q, slots_k=sk, slots_v=sv, grad_out=go), res,
          dict(rounds=3, causal=0, dtype="float32"))

    # 2. Same shape with a loss on the last-round weights too (exercises grad_weights).
    g = torch.Generator().manual_seed(1)
    q = _randn(g, 1, 2, 96, 64)
    sk = _randn(g, 1, 2, 64, 64)
    sv = _randn(g, 1, 2, 64, 64, std=0.5)
    go = _randn(g, 1, 2, 96, 64)
    gw = _randn(g, 1, 2, 96, 7)
    res = compose(ref, q, sk, sv, 2, False, grad_out=go, grad_w=gw)
    _save("weights_grad", dict(q=q, slots_k=sk, slots_v=sv, grad_out=go, grad_w=gw), res,
          dict(rounds=2, causal=0, dtype="float32"))

    # 3. Causal, small M and d (ragged sizes), fwd + bwd.
    g = torch.Generator().manual_seed(2)
    q = _randn(g, 1, 3, 77, 32)
    sk = _randn(g, 1, 3, 48, 32)
    sv = _randn(g, 1, 3, 48, 32, std=0.3)
    go = _randn(g, 1, 3, 77, 32)
    res = compose(ref, q, sk, sv, 3, True, grad_out=go)
    _save("causal_small", dict(q=q, slots_k=sk, slots_v=sv, grad_out=go), res,
          dict(rounds=3, causal=1, dtype="float32"))

    # 4. fp16-representable inputs (configs[1] distribution, reduced size).
    g = torch.Generator().manual_seed(3)
    q = _randn(g, 1, 2, 256, 64, dtype=torch.float16)
    sk = _randn(g, 1, 2, 256, 64, dtype=torch.float16)
    sv = torch.zeros(1, 2, 256, 64)
    go = _randn(g, 1, 2, 256, 64, dtype=torch.float16)
    res = compose(ref, q, sk, sv, 3, False, grad_out=go)
    _save("fp16_inputs", dict(q=q, slots_k=sk, slots_v=sv, grad_out=go), res,
          dict(rounds=3, causal=0, dtype="float16"))

    # 5. bf16-representable causal inputs (configs[2] distribution, reduced size).
    g = torch.Generator().manual_seed(4)
    q = _randn(g, 1, 2, 256, 64, dtype=torch.bfloat16)
    sk = _randn(g, 1, 2, 256, 64, std=1.0 / 8.0, dtype=torch.bfloat16)
    sv = _randn(g, 1, 2, 256, 64, std=0.02, dtype=torch.bfloat16)
    go = _randn(g, 1, 2, 256, 64, dtype=torch.bfloat16)
    res = compose(ref, q, sk, sv, 3, True, grad_out=go)
    _save("bf16_causal", dict(q=q, slots_k=sk, slots_v=sv, grad_out=go), res,
          dict(rounds=3, causal=1, dtype="bfloat16"))

    # 6. The reference's own round loop (slot_murmurate_reference, reference.py:138-191)
    #    with x = 0 and q_proj = k_proj = v_proj: pins the north-star composition.
    g = torch.Generator().manual_seed(5)
    B, N, H, Dh, M = 2, 64, 4, 16, 32
    qp = _randn(g, B, N, H * Dh)
    ske = _randn(g, H, M, Dh)
    sve = _randn(g, H, M, Dh, std=0.5)
    out6 = ref.slot_murmurate_reference(torch.zeros(B, N, H * Dh), qp, qp, qp, ske, sve,
                                        num_heads=H, rounds=3)
    _save("reference_loop", dict(q_proj=qp, slot_k_emb=ske, slot_v_emb=sve),
          dict(out=out6), dict(rounds=3, heads=H))

    # 7. Standalone phases on random indices/weights (reference tests' shapes).
    g = torch.Generator().manual_seed(6)
    tk = _randn(g, 1, 2, 16, 16)
    tv = _randn(g, 1, 2, 16, 16)
    sk = _randn(g, 1, 2, 64, 16)
    sv = _randn(g, 1, 2, 64, 16)
    idx = torch.randint(0, 64, (1, 2, 16, 7), generator=g)
    w = torch.rand(1, 2, 16, 7, generator=g)
    w = w / w.sum(-1, keepdim=True)
    nk, nv = ref.slot_update_reference(tk, tv, sk, sv, idx, w, 0.9)
    dk, dv = ref.slot_diffusion_reference(sk, sv, 0.1)
    _save("phases", dict(tk=tk, tv=tv, slots_k=sk, slots_v=sv, idx=idx, w=w),
          dict(upd_k=nk, upd_v=nv, diff_k=dk, diff_v=dv), dict(alpha=0.9, gamma=0.1))

    make_surface(ref)


def surface_bias_fn(M: int):
    """The position-bias function of the ``surface`` fixture (also used by the tests):
    depends on the current residual stream, so it changes every round."""
    ramp = torch.linspace(-1.0, 1.0, M)
    return lambda xh: 0.1 * torch.tanh(xh[..., :1]) * ramp.to(xh.device, xh.dtype)


def make_surface(ref):
    """8. The full op surface (reference.py:138-191): residual x, separate q/k/v
    projections, a selection mask, a position bias from x, dynamic M (N=64 -> 32 of
    the 48 slots active), with gradients of every input. Every row keeps at least 8
    selectable slots, so torch.topk has no ties to order."""
    g = torch.Generator().manual_seed(8)
    B, N, H, Dh, M = 2, 64, 2, 16, 48
    x = _randn(g, B, N, H * Dh)
    qp, kp, vp = (_randn(g, B, N, H * Dh) for _ in range(3))
    ske = _randn(g, H, M, Dh)
    sve = _randn(g, H, M, Dh, std=0.5)
    mask = (torch.rand(N, M, generator=g) > 0.15).to(torch.uint8)
    assert int(mask[:, :32].sum(-1).min()) >= 8
    go = _randn(g, B, N, H * Dh)
    leaves = [t.clone().requires_grad_(True) for t in (x, qp, kp, vp, ske, sve)]
    out = ref.slot_murmurate_reference(*leaves, num_heads=H, rounds=3, mask=mask,
                                       position_bias_fn=surface_bias_fn(M), use_dynamic_m=True)
    (out * go).sum().backward()
    names = ("x", "q_proj", "k_proj", "v_proj", "slot_k_emb", "slot_v_emb")
    res = dict(out=out.detach(), **{"grad_" + n: t.grad for n, t in zip(names, leaves)})
    _save("surface", dict(x=x, q_proj=qp, k_proj=kp, v_proj=vp, slot_k_emb=ske, slot_v_emb=sve,
                          mask=mask.to(torch.int64), grad_out=go), res,
          dict(rounds=3, heads=H, use_dynamic_m=1))


if __name__ == "__main__":
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MURM_REFERENCE_SRC")
    if not src:
        sys.exit("usage: make_golden.py /path/to/reference/src  (or set MURM_REFERENCE_SRC)")
    main(src)
