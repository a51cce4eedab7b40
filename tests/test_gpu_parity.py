"""GPU parity of slot_murmurate (CUDA path through the C ABI) against the oracle.

Protocol (fixed here, applied to every case; helpers in tests/parity.py):
- reference fixtures: indices equal on every row, out / weights / all gradients within tolerance;
- seeded cases: the GPU's per-round picks are forced into the oracle, so out, weights and all
  gradients are compared on every row (none skipped); the picks must equal the oracle's own
  top-7 on every row whose top-8 scores are unambiguous (adjacent gaps > 1e-5 * max|score|,
  oracle.row_gap_ok), and the oracle's fp32 slot state of every round, handed to the GPU, must
  give the oracle's indices on those rows too (differing near-tie rows are counted and bounded);
- fp32: within atol 1e-4, rtol 1e-4; fp16 / bf16: within atol 2e-3, rtol 1e-2 (fp32
  accumulation everywhere).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from oracle import murmurate as om
from parity import gpu_run, protocol_a, protocol_b

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = {torch.float32: dict(atol=1e-4, rtol=1e-4),
       torch.float16: dict(atol=2e-3, rtol=1e-2),
       torch.bfloat16: dict(atol=2e-3, rtol=1e-2)}


def _op():
    from murmurative_attention_b200 import slot_murmurate
    return slot_murmurate


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: (torch.from_numpy(z[k]) if z[k].dtype.kind != "U" else str(z[k])) for k in z.files}


def run_gpu(q, sk, sv, rounds, causal, grad_out=None, grad_w=None):
    dev = torch.device("cuda")
    qd = q.detach().to(dev).requires_grad_(grad_out is not None)
    skd = sk.detach().to(dev).requires_grad_(grad_out is not None)
    svd = sv.detach().to(dev).requires_grad_(grad_out is not None)
    out, idx, w = _op()(qd, skd, svd, rounds=rounds, causal=causal)
    res = dict(out=out.detach().float().cpu(), idx=idx.cpu(), w=w.detach().cpu())
    if grad_out is not None:
        loss = (out.float() * grad_out.to(dev).float()).sum()
        if grad_w is not None:
            loss = loss + (w * grad_w.to(dev).float()).sum()
        loss.backward()
        res.update(grad_q=qd.grad.float().cpu(), grad_sk=skd.grad.float().cpu(), grad_sv=svd.grad.float().cpu())
    return res


def compare(res, ref, dtype):
    """Every row's indices equal; out, weights and (when present) all gradients within tolerance."""
    tol = TOL[dtype]
    mism = (res["idx"] != ref["idx"]).any(-1)
    assert not mism.any(), f"{int(mism.sum())} rows have different indices"
    torch.testing.assert_close(res["out"], ref["out"].float(), **tol)
    torch.testing.assert_close(res["w"], ref["w"].float(), **tol)
    if "grad_q" in ref:
        for k in ("grad_q", "grad_sk", "grad_sv"):
            torch.testing.assert_close(res[k], ref[k].float(), **tol, msg=lambda m, k=k: f"{k}: {m}")


DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


@pytest.mark.parametrize("name", ["config1", "weights_grad", "causal_small", "fp16_inputs", "bf16_causal"])
def test_matches_reference_fixture(name):
    """GPU output against outputs of the reference implementation itself."""
    f = load(name)
    dt = DTYPES[f["meta_dtype"]]
    q, sk, sv, go = (f[k].to(dt) for k in ("q", "slots_k", "slots_v", "grad_out"))
    res = run_gpu(q, sk, sv, int(f["meta_rounds"]), bool(int(f["meta_causal"])), go, f.get("grad_w"))
    ref = dict(out=f["out"], idx=f["idx"].long(), w=f["w"], grad_q=f["grad_q"], grad_sk=f["grad_sk"],
               grad_sv=f["grad_sv"])
    compare(res, ref, dt)


CASES = [
    # B, H, N, D, M, R, causal, dtype
    (1, 2, 128, 64, 256, 3, False, torch.float32),
    (2, 3, 77, 32, 48, 3, True, torch.float32),
    (1, 1, 1, 16, 7, 2, False, torch.float32),      # single token, minimum slots
    (1, 2, 300, 16, 16, 4, True, torch.float32),    # ragged N, M < tile
    (1, 2, 256, 64, 256, 1, True, torch.float16),
    (2, 2, 200, 64, 128, 3, False, torch.bfloat16),
    (1, 4, 520, 64, 256, 3, True, torch.bfloat16),
    (1, 2, 40, 64, 9, 2, True, torch.float16),      # tensor-core path, causal, M < 13 (rows n < 6 pick masked slots)
    (1, 1, 20, 64, 7, 3, True, torch.bfloat16),     # tensor-core path, causal, minimum slots
    # more (b,h) x tile units than SMs: forward CTAs whose runs span pairs (several segments
    # per CTA, a pair's slot sums from partials of two CTAs)
    (1, 150, 256, 64, 64, 2, False, torch.float16),   # runs of 3 tiles: 2 of one pair + 1 of the next
    (2, 80, 128, 64, 32, 3, True, torch.float16),     # one tile per pair: 2 whole pairs per CTA
]


@pytest.mark.parametrize("B,H,N,D,M,R,causal,dt", CASES)
def test_matches_oracle_seeded(B, H, N, D, M, R, causal, dt):
    g = torch.Generator().manual_seed(B * 1000 + N + M + R)
    q = torch.randn(B, H, N, D, generator=g).to(dt)
    sk = torch.randn(B, H, M, D, generator=g).to(dt)
    sv = (torch.randn(B, H, M, D, generator=g) * 0.3).to(dt)
    go = torch.randn(B, H, N, D, generator=g).to(dt)
    gw = torch.randn(B, H, N, 7, generator=g)
    protocol_a(q, sk, sv, R, causal, tol=TOL[dt])
    res = gpu_run(q, sk, sv, R, causal, go, gw)
    protocol_b(q, sk, sv, R, causal, res, go, gw, tol=TOL[dt])


@pytest.mark.parametrize("gscale", [1.0, 512.0])
def test_bf16_backward_operand_paths(gscale):
    """The bf16 backward's scatter operands: q and grad_out tiles as fp16 under the pair's
    power-of-two scales while their largest magnitudes stay within 2^8 (gscale 1), two bf16 terms
    per weight and coefficient beyond that (gscale 512: grad_out up to ~2500). The backward is
    linear in grad_out and the weights' gradient, so the GPU's gradients for the scaled ones,
    divided by the (power-of-two) scale, are compared with the oracle's for the unscaled ones."""
    g = torch.Generator().manual_seed(4242)
    B, H, N, M, R = 1, 3, 640, 128, 3
    q = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16)
    sk = torch.randn(B, H, M, 64, generator=g).to(torch.bfloat16)
    sv = (torch.randn(B, H, M, 64, generator=g) * 0.3).to(torch.bfloat16)
    go = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16)
    gw = torch.randn(B, H, N, 7, generator=g)
    res = gpu_run(q, sk, sv, R, True, (go.float() * gscale).to(torch.bfloat16), gw * gscale)
    for k in ("grad_q", "grad_sk", "grad_sv"):
        res[k] = res[k] / gscale
    protocol_b(q, sk, sv, R, True, res, go, gw, tol=TOL[torch.bfloat16])


@pytest.mark.parametrize("B,H,N,M,causal", [(1, 150, 256, 64, False)])
def test_forward_runs_spanning_pairs_bf16(B, H, N, M, causal):
    """bf16 forward where every CTA's run spans two (b,h) pairs: out / indices / weights. Cases of
    ~1M elements put single bf16 elements at the edge of the 2e-3 tolerance (the attend output and
    the backward's slot tables are one 16-bit term each; the split changes neither), so gradients
    and the causal variant of the spanning runs are checked in fp16 above."""
    g = torch.Generator().manual_seed(B * 1000 + N + M)
    q = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16)
    sk = torch.randn(B, H, M, 64, generator=g).to(torch.bfloat16)
    sv = (torch.randn(B, H, M, 64, generator=g) * 0.3).to(torch.bfloat16)
    res = gpu_run(q, sk, sv, 3, causal)
    protocol_b(q, sk, sv, 3, causal, res)


def test_rounds_zero_gives_zero():
    q = torch.randn(1, 2, 64, 32, device="cuda")
    s = torch.randn(1, 2, 16, 32, device="cuda")
    out, idx, w = _op()(q, s, s, rounds=0)
    assert out.abs().max().item() == 0 and idx.abs().max().item() == 0


def test_deterministic_bitwise():
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(2, 4, 1000, 64, device="cuda", generator=g).half().requires_grad_(True)
    sk = torch.randn(2, 4, 256, 64, device="cuda", generator=g).half().requires_grad_(True)
    sv = torch.zeros(2, 4, 256, 64, device="cuda").half().requires_grad_(True)
    go = torch.randn(2, 4, 1000, 64, device="cuda", generator=g).half()
    outs = []
    for _ in range(2):
        q.grad = sk.grad = sv.grad = None
        out, idx, w = _op()(q, sk, sv, rounds=3)
        out.backward(go)
        outs.append([t.detach().clone() for t in (out, idx, w, q.grad, sk.grad, sv.grad)])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_strided_q_and_broadcast_slots():
    """q as the transposed view of a [B,N,H,d] projection and slots expanded over
    the batch are read in place and give the same result as contiguous copies."""
    g = torch.Generator(device="cuda").manual_seed(4)
    B, N, H, D, M = 2, 130, 4, 64, 64
    x = torch.randn(B, N, H * D, device="cuda", generator=g)
    q = x.view(B, N, H, D).transpose(1, 2)
    emb = torch.randn(H, M, D, device="cuda", generator=g)
    sk = emb.unsqueeze(0).expand(B, -1, -1, -1)
    sv = torch.zeros_like(sk)
    q1 = q.detach().requires_grad_(True)
    sk1 = emb.detach().clone().requires_grad_(True)
    o1, i1, w1 = _op()(q1, sk1.unsqueeze(0).expand(B, -1, -1, -1), sv, rounds=3)
    q2 = q.detach().contiguous().requires_grad_(True)
    sk2 = emb.detach().clone().requires_grad_(True)
    o2, i2, w2 = _op()(q2, sk2.unsqueeze(0).expand(B, -1, -1, -1).contiguous(), sv.contiguous(), rounds=3)
    assert o1.stride() == q.stride()  # output written in the projection's layout
    assert torch.equal(i1, i2) and torch.equal(w1, w2) and torch.equal(o1, o2)
    go = torch.randn_like(o2)
    o1.backward(go)
    o2.backward(go)
    assert torch.equal(q1.grad, q2.grad) and torch.equal(sk1.grad, sk2.grad)


def test_errors_mirror_reference():
    op = _op()
    q = torch.randn(1, 1, 8, 16, device="cuda")
    s = torch.randn(1, 1, 16, 16, device="cuda")
    with pytest.raises(TypeError):
        op(q.double(), s.double(), s.double())
    with pytest.raises(ValueError):
        op(q, s, s, top_k=5)
    with pytest.raises(RuntimeError):
        op(q, s[:, :, :6], s[:, :, :6])        # fewer slots than picks
    with pytest.raises(RuntimeError):
        op(q.cpu(), s.cpu(), s.cpu())


@pytest.mark.parametrize("dt,causal,N,M", [(torch.float16, False, 1000, 256), (torch.bfloat16, True, 700, 256),
                                           (torch.float16, True, 129, 96), (torch.bfloat16, False, 64, 7)])
def test_tensor_core_forward_matches_cuda_core_forward(dt, causal, N, M, monkeypatch):
    """The tcgen05 forward (fp16/bf16, d=64) and the fp32 CUDA-core forward agree:
    indices on every unambiguous row, out/weights within the 16-bit tolerance."""
    from murmurative_attention_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(N + M)
    q = torch.randn(2, 3, N, 64, device="cuda", generator=g).to(dt)
    sk = torch.randn(2, 3, M, 64, device="cuda", generator=g).to(dt)
    sv = (torch.randn(2, 3, M, 64, device="cuda", generator=g) * 0.2).to(dt)
    o_tc, i_tc, w_tc = _op()(q, sk, sv, rounds=3, causal=causal)
    _lib.device_status()
    monkeypatch.setenv("MURM_FORCE_SIMT", "1")
    o_s, i_s, w_s = _op()(q, sk, sv, rounds=3, causal=causal)
    _lib.device_status()
    tr = oracle.slot_murmurate_trace(q.float().cpu(), sk.float().cpu(), sv.float().cpu(), 3, causal)
    ok = om.row_gap_ok(tr["top8"][-1])
    mism = (i_tc.cpu() != i_s.cpu()).any(-1)
    assert not (mism & ok).any(), f"{int((mism & ok).sum())} unambiguous rows differ"
    keep = ~mism
    torch.testing.assert_close(o_tc.float().cpu()[keep], o_s.float().cpu()[keep], atol=2e-3, rtol=1e-2)
    torch.testing.assert_close(w_tc.cpu()[keep], w_s.cpu()[keep], atol=2e-3, rtol=1e-2)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two CUDA devices")
def test_two_devices_in_one_process():
    """The kernels' shared-memory opt-ins belong to each device's context: a forward on cuda:1
    after one on cuda:0 in the same process launches (tensor-core and CUDA-core paths) and gives
    the same result. Plain kernels on each device; no peer memory."""
    g = torch.Generator().manual_seed(9)
    for dt in (torch.float16, torch.float32):
        q = torch.randn(1, 4, 512, 64, generator=g).to(dt)
        sk = torch.randn(1, 4, 256, 64, generator=g).to(dt)
        sv = torch.zeros(1, 4, 256, 64).to(dt)
        res = []
        for d in (0, 1):
            dev = torch.device("cuda", d)
            with torch.cuda.device(dev):
                out, idx, w = _op()(q.to(dev), sk.to(dev), sv.to(dev), rounds=3)
                torch.cuda.synchronize(dev)
            res.append((out.cpu(), idx.cpu(), w.cpu()))
        for a, b in zip(*res):
            assert torch.equal(a, b)
