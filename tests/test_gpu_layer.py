"""MurmurativeAttention layer (README.md:82-102; BASELINE config 4's module) on the GPU
against the oracle composition in fp32 on the CPU.

The oracle is fed the layer's own 16-bit q projection (recomputed with the same GEMM), so
both sides select the same slots and the comparison measures the layer's wiring and
precision: head split, the op, o_proj, and the gradients of q_proj, o_proj and the slot
embeddings. Tolerances are relative Frobenius errors for 16-bit GEMMs with fp32
accumulation.
"""
import pytest
import torch

from murmurative_attention_b200 import MurmurativeAttention
from oracle import murmurate as orc

pytestmark = pytest.mark.gpu

REL = {torch.float16: 1e-2, torch.bfloat16: 3e-2}


def rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
def test_layer_forward_backward_matches_oracle(dtype, causal):
    torch.manual_seed(0)
    dim, heads, slots, N, B = 128, 2, 64, 256, 2
    layer = MurmurativeAttention(dim, heads, slots, rounds=3, causal=causal).cuda().to(dtype)
    with torch.no_grad():  # config 4's initialisation: projections ~ N(0, 1/dim)
        layer.q_proj.weight.normal_(0.0, dim ** -0.5)
        layer.o_proj.weight.normal_(0.0, dim ** -0.5)
    x = torch.randn(B, N, dim, device="cuda", dtype=dtype)
    y = layer(x)
    gy = torch.randn_like(y)
    y.backward(gy)

    # oracle: the same 16-bit q, then the op, o_proj and all gradients in fp32
    with torch.no_grad():
        q16 = layer.q_proj(x)
    xc = x.float().cpu()
    q = q16.float().cpu().view(B, N, heads, dim // heads).transpose(1, 2).contiguous().requires_grad_()
    emb = layer.slot_embeddings.detach().float().cpu().requires_grad_()
    wo = layer.o_proj.weight.detach().float().cpu().requires_grad_()
    sk = emb.unsqueeze(0).expand(B, -1, -1, -1)
    o, _, _ = orc.slot_murmurate(q, sk, torch.zeros_like(sk), rounds=3, causal=causal)
    yr = o.transpose(1, 2).reshape(B, N, dim) @ wo.t()
    yr.backward(gy.float().cpu())
    dq = q.grad.transpose(1, 2).reshape(B * N, dim)
    dwq = dq.t() @ xc.reshape(B * N, dim)

    tol = REL[dtype]
    assert rel(y, yr) < tol
    assert rel(layer.o_proj.weight.grad, wo.grad) < tol
    assert rel(layer.slot_embeddings.grad, emb.grad) < tol
    assert rel(layer.q_proj.weight.grad, dwq) < tol
