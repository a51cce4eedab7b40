"""Streaming decode (murmurative_attention_b200.decode, ``murm_decode_step``) against the
oracle composition of the reference's phases with one token per step, as the
reference's decode plan writes it (docs/murmurative-attention-kernel-plan.md:154-173):
select (slots above the token's absolute position masked) -> attend -> residual ->
update with the token -> diffusion, the pool carried from step to step.
"""
import pytest
import torch

from murmurative_attention_b200 import functional as F
from murmurative_attention_b200.decode import SlotPool
from oracle import murmurate as om

pytestmark = pytest.mark.gpu


def oracle_step(sk, sv, q, k, v, x, pos, alpha, gamma, causal=True):
    """One decode step of the reference phases on [B, H, 1, d] tensors."""
    B, H, M, D = sk.shape
    mask = None
    if causal:
        mask = (torch.arange(M).view(1, 1, 1, M) <= pos.view(B, 1, 1, 1)).to(torch.uint8)
    scores = om.slot_scores(q.float(), sk.float(), mask=mask)
    idx = om.topk_indices(scores)
    ok = om.row_gap_ok(torch.sort(scores, dim=-1, descending=True).values[..., :8])
    o, w = om.slot_attend(q.float(), sk.float(), sv.float(), idx)
    out = x.float() + o
    nk, nv = om.slot_update(k, v, sk, sv, idx, w, alpha)
    nk, nv = om.slot_diffusion(nk, nv, gamma)
    return out, nk, nv, idx, ok


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_decode_steps_match_oracle(dt):
    g = torch.Generator().manual_seed(21)
    B, H, M, D, T = 2, 3, 64, 32, 24
    alpha, gamma = 0.9, 0.1
    ske = (torch.randn(H, M, D, generator=g)).to(dt)
    sve = (torch.randn(H, M, D, generator=g) * 0.5).to(dt)
    pool = SlotPool.from_embeddings(ske.cuda(), sve.cuda(), B)
    sk = ske.unsqueeze(0).expand(B, -1, -1, -1).clone()
    sv = sve.unsqueeze(0).expand(B, -1, -1, -1).clone()
    pos = torch.zeros(B, dtype=torch.int64)
    tol = dict(atol=1e-5, rtol=1e-5) if dt == torch.float32 else dict(atol=3e-3, rtol=1e-2)
    for t in range(T):
        q, k, v, x = (torch.randn(B, H, D, generator=g).to(dt) for _ in range(4))
        out, idx, w = pool.step(q.cuda(), k.cuda(), v.cuda(), x.cuda(), causal=True, alpha=alpha, gamma=gamma,
                                return_selection=True)
        ro, sk, sv, ridx, ok = oracle_step(sk, sv, q.unsqueeze(2), k.unsqueeze(2), v.unsqueeze(2),
                                           x.unsqueeze(2), pos, alpha, gamma)
        pos += 1
        ok = ok[..., 0]
        assert torch.equal(idx.cpu()[ok], ridx[..., 0, :][ok]), f"step {t}"
        if bool(ok.all()):
            torch.testing.assert_close(out.float().cpu(), ro[..., 0, :], **tol)
        # carry the kernel's own pool forward (the oracle's may differ by rounding)
        sk, sv = pool.keys.cpu().clone(), pool.values.cpu().clone()
    assert torch.equal(pool.positions.cpu(), torch.full((B,), T, dtype=torch.int64))


def test_decode_pool_update_matches_oracle_fp32():
    """The pool after one step equals the oracle's update + diffusion."""
    g = torch.Generator().manual_seed(22)
    B, H, M, D = 1, 2, 48, 64
    sk, sv = torch.randn(B, H, M, D, generator=g), torch.randn(B, H, M, D, generator=g)
    pool = SlotPool(sk.cuda(), sv.cuda(), positions=torch.tensor([40]))
    q, k, v = (torch.randn(B, H * D, generator=g) for _ in range(3))
    out = pool.step(q.cuda(), k.cuda(), v.cuda(), causal=True, gamma=0.15)
    ro, nk, nv, _, ok = oracle_step(sk, sv, q.view(B, H, 1, D), k.view(B, H, 1, D), v.view(B, H, 1, D),
                                    torch.zeros(B, H, 1, D), torch.tensor([40]), 0.9, 0.15)
    assert bool(ok.all())
    torch.testing.assert_close(out.cpu(), ro[..., 0, :].reshape(B, H * D), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(pool.keys.cpu(), nk, atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(pool.values.cpu(), nv, atol=1e-6, rtol=1e-6)


def test_prefill_then_decode():
    """Prefill with the full op (return_slots) and continue token by token."""
    g = torch.Generator().manual_seed(23)
    B, N, H, Dh, M = 1, 40, 2, 16, 32
    ins = [torch.randn(B, N, H * Dh, generator=g) for _ in range(4)]
    ske, sve = torch.randn(H, M, Dh, generator=g), torch.randn(H, M, Dh, generator=g) * 0.5
    out, sk, sv = F.slot_murmurate(*[t.cuda() for t in ins], ske.cuda(), sve.cuda(), num_heads=H, rounds=3,
                                   causal=True, use_dynamic_m=False, return_slots=True)
    ref = om.slot_murmurate_full(*ins, ske, sve, num_heads=H, rounds=3, causal=True)
    torch.testing.assert_close(out.cpu(), ref, atol=1e-4, rtol=1e-4)
    pool = SlotPool(sk, sv, positions=torch.full((B,), N))
    q, k, v, x = (torch.randn(B, H * Dh, generator=g) for _ in range(4))
    y = pool.step(q.cuda(), k.cuda(), v.cuda(), x.cuda(), causal=True)
    assert y.shape == (B, H * Dh) and bool(torch.isfinite(y).all())
    assert int(pool.positions[0]) == N + 1
