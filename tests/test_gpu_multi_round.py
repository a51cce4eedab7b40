"""The tensor-core forward runs all rounds in one cooperative launch: between rounds, the CTAs
whose runs end in a (b,h) pair combine its slot-sum partials (token order), apply the EMA and the
diffusion and write the next round's state and operand images, and a pair's next round starts
once its own finalize is done. The fallback is one launch per round with a separate finalize
kernel (MURM_FWD_LAUNCH_PER_ROUND=1). Both add the same partials in the same order with the same
rounded operations, so outputs, round records and gradients must be bitwise equal; the cases
cover CTA runs that span pairs, pairs covered by one CTA that runs on into the next pair (that
CTA finalizes them alone), ragged tiles, causal masking and bf16.
"""
import pytest
import torch

from murmurative_attention_b200 import _lib, slot_murmurate

pytestmark = pytest.mark.gpu

CASES = [
    # B, H, N, M, R, causal, dtype
    (1, 16, 2048, 256, 3, False, torch.float16),
    (1, 150, 256, 64, 2, False, torch.float16),   # runs of 3 tiles: 2 of one pair + 1 of the next
    (2, 80, 128, 32, 3, True, torch.float16),     # one tile per pair: CTAs finalize whole pairs alone
    (1, 3, 1000, 100, 4, True, torch.float16),    # ragged last tile, M < 256
    (1, 4, 520, 256, 3, True, torch.bfloat16),
]


def _run(q, sk, sv, go, R, causal):
    qd, skd, svd = (t.cuda().requires_grad_(True) for t in (q, sk, sv))
    out, idx, w = slot_murmurate(qd, skd, svd, rounds=R, causal=causal)
    ((out.float() * go.cuda().float()).sum() + w.sum()).backward()
    _lib.device_status()
    return [t.detach().cpu() for t in (out, idx, w, qd.grad, skd.grad, svd.grad)]


@pytest.mark.parametrize("B,H,N,M,R,causal,dt", CASES)
def test_one_launch_equals_launch_per_round(B, H, N, M, R, causal, dt, monkeypatch):
    g = torch.Generator().manual_seed(7 * N + M + R)
    q = torch.randn(B, H, N, 64, generator=g).to(dt)
    sk = torch.randn(B, H, M, 64, generator=g).to(dt)
    sv = (torch.randn(B, H, M, 64, generator=g) * 0.3).to(dt)
    go = torch.randn(B, H, N, 64, generator=g).to(dt)
    monkeypatch.delenv("MURM_FWD_LAUNCH_PER_ROUND", raising=False)
    one = _run(q, sk, sv, go, R, causal)
    monkeypatch.setenv("MURM_FWD_LAUNCH_PER_ROUND", "1")
    per = _run(q, sk, sv, go, R, causal)
    for name, a, b in zip(("out", "indices", "weights", "grad_q", "grad_slots_k", "grad_slots_v"), one, per):
        assert torch.equal(a, b), name


def test_one_launch_per_forward():
    """The R rounds of the forward are one launch of the round kernel (plus the round-0 load)."""
    B, H, N, M = 1, 8, 1024, 128
    q = torch.randn(B, H, N, 64, device="cuda", dtype=torch.float16)
    sk = torch.randn(B, H, M, 64, device="cuda", dtype=torch.float16)
    sv = torch.randn(B, H, M, 64, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        slot_murmurate(q, sk, sv, rounds=3)
        torch.cuda.synchronize()
        n0 = _lib.kernel_launches()
        slot_murmurate(q, sk, sv, rounds=3)
        torch.cuda.synchronize()
    assert _lib.kernel_launches() - n0 == 2
