"""Parity helpers shared by the GPU tests (not a test module).

Two protocols compare the CUDA path (through the C ABI) with the CPU oracle on every round of
the reference's loop (reference.py:177-189):

A. Oracle-led, teacher-forced: the oracle's fp32 slot state entering round r is handed to the
   GPU (murm_slot_murmurate_fwd_f32_slots, one round); its indices must equal the oracle's on
   every row whose top-8 scores are unambiguous (adjacent gaps > 1e-5 * max|score|,
   oracle.row_gap_ok); differing near-tie rows are counted, printed and bounded.
B. GPU-led: the GPU's own per-round indices are forced into the oracle
   (oracle.slot_murmurate_forced), so out, weights and every gradient are compared on every row
   (no row or gradient is skipped because of a near tie); the GPU's picks must equal the
   oracle's own top-7 on every unambiguous row of the state that followed them.

Tolerances. out, weights and grad_q: atol + rtol * |ref| elementwise (fp16 / bf16: 2e-3, 1e-2;
fp32: 1e-4, 1e-4). The slot gradients are sums over every (token, pick) that chose the slot,
in every round: up to ~2e4 terms per slot and round at N = 65536, where "hub" slots (the
diffusion boundaries 0 and M-1 attract the most picks) collect thousands. Their tensor-core
path takes 16-bit operands for those sums (the weights of the dV scatter in fp16, the slot
tables of the softmax adjoint in bf16), each rounded with relative error <= u (2^-11 fp16,
2^-8 bf16), so the forward error of such a sum is of order u * rho, with rho the root sum of
squares of its terms (independent roundings). The slot-gradient tolerance adds that term:
atol + rtol * |ref| + 2 * u * rho, rho from the oracle's own terms: scale * da * q scattered into
dK (da = the softmax adjoint of the round) and w * G into dV, summed in squares over the rounds.
"""
import ctypes

import torch

import oracle
from murmurative_attention_b200 import _lib, ops
from murmurative_attention_b200 import slot_murmurate

TOL16 = dict(atol=2e-3, rtol=1e-2)   # fp16 / bf16: the north-star's stated tolerance
TOL32 = dict(atol=1e-4, rtol=1e-4)   # fp32
MAX_TIE_FRACTION = 1e-4  # differing near-tie rows allowed per round, as a fraction of all rows


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def gpu_round_from_state(q, K, V, causal):
    """One round from fp32 slot state K, V [B,H,M,d] (oracle-led teacher forcing): indices,
    weights and the round's attend output."""
    lib = _lib.load_library()
    dev = torch.device("cuda")
    qd = q.to(dev).contiguous()
    Kd = K.to(dev, torch.float32).contiguous()
    Vd = V.to(dev, torch.float32).contiguous()
    shape = ops._make_shape(qd, Kd.shape[2], 1, 7, causal, 0.9, 0.15, None)
    saved_b, fws_b, _ = ops.slot_murmurate_sizes(shape)
    B, H, N, _ = qd.shape
    out = torch.empty_like(qd)
    idx = torch.empty(B, H, N, 7, dtype=torch.int64, device=dev)
    w = torch.empty(B, H, N, 7, dtype=torch.float32, device=dev)
    saved = torch.empty(saved_b, dtype=torch.uint8, device=dev)
    ws = torch.empty(fws_b, dtype=torch.uint8, device=dev)
    S = ops._strides
    a = _lib.FwdArgs(shape, qd.data_ptr(), S(qd), Kd.data_ptr(), S(Kd), Vd.data_ptr(), S(Vd), out.data_ptr(),
                     S(out), idx.data_ptr(), w.data_ptr(), saved.data_ptr(), saved_b, ws.data_ptr(), fws_b)
    _lib.check(lib.murm_slot_murmurate_fwd_f32_slots(ctypes.byref(a), _stream()))
    _lib.device_status()
    return idx.cpu(), w.cpu(), out.float().cpu()


def gpu_run(q, sk, sv, rounds, causal, go=None, gw=None):
    """The op through ops.slot_murmurate (C ABI): per-round indices, and out, weights and
    gradients of the full R-round call."""
    dev = torch.device("cuda")
    with torch.no_grad():
        per_round = []
        for r in range(1, rounds + 1):
            _, i_r, _ = slot_murmurate(q.to(dev), sk.to(dev), sv.to(dev), rounds=r, causal=causal)
            per_round.append(i_r.cpu())
    need_grad = go is not None
    qd, skd, svd = (t.detach().to(dev).requires_grad_(need_grad) for t in (q, sk, sv))
    out, idx, w = slot_murmurate(qd, skd, svd, rounds=rounds, causal=causal)
    res = dict(out=out.detach().float().cpu(), idx=idx.cpu(), w=w.detach().cpu(), per_round=per_round)
    if need_grad:
        loss = (out.float() * go.to(dev).float()).sum() + (w * gw.to(dev)).sum()
        loss.backward()
        res.update(grad_q=qd.grad.float().cpu(), grad_sk=skd.grad.float().cpu(), grad_sv=svd.grad.float().cpu())
    _lib.device_status()
    assert torch.equal(res["per_round"][-1], res["idx"])
    return res


def check_indices(got, ref_idx, top8, label):
    """Indices equal on every unambiguous row; returns (differing near-tie rows, ambiguous rows)."""
    ok = oracle.row_gap_ok(top8)
    diff = (got != ref_idx).any(-1)
    bad = diff & ok
    assert not bad.any(), f"{label}: {int(bad.sum())} unambiguous rows differ from the oracle's top-7"
    nd, na, rows = int(diff.sum()), int((~ok).sum()), diff.numel()
    print(f"{label}: {nd} near-tie rows differ, {na} ambiguous rows, of {rows}")
    assert nd <= max(1, MAX_TIE_FRACTION * rows), f"{label}: {nd} differing near-tie rows"
    return nd, na


def protocol_a(q, sk, sv, rounds, causal, tol=TOL16):
    """Oracle-led: every round from the oracle's own fp32 state."""
    tr = oracle.slot_murmurate_trace(q.float(), sk.float(), sv.float(), rounds, causal)
    for r in range(rounds):
        idx, w, out = gpu_round_from_state(q, tr["K"][r], tr["V"][r], causal)
        check_indices(idx, tr["idx"][r], tr["top8"][r], f"A round {r}")
        same = (idx == tr["idx"][r]).all(-1)
        torch.testing.assert_close(w[same], tr["w"][r][same], **tol)
        if r == 0:  # round 0's attend output alone is the oracle's first summand
            o0, _ = oracle.slot_attend(q.float(), tr["K"][0], tr["V"][0], tr["idx"][0])
            torch.testing.assert_close(out[same], o0[same], **tol)


UNIT_ROUNDOFF = {torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8, torch.float32: 2.0 ** -24}


def slot_grad_rho(q, go, forced, info, M, scale=None):
    """Root sum of squares of the terms each slot-gradient entry sums, from the forced oracle's
    rounds (after its backward pass): scale * da * q into dK and w * G into dV."""
    qf = q.detach().float()
    G = go.float()
    B, H, N, D = qf.shape
    sc = scale if scale is not None else 1.0 / (D ** 0.5)
    rk = torch.zeros(B, H, M, D)
    rv = torch.zeros(B, H, M, D)
    for idx, w, lg in zip(forced, info["w"], info["logits"]):
        da = lg.grad
        where = idx.reshape(B, H, N * 7, 1).expand(-1, -1, -1, D)
        tk = (sc * da).unsqueeze(-1) * qf.unsqueeze(-2)
        tv = w.detach().unsqueeze(-1) * G.unsqueeze(-2)
        rk.scatter_add_(2, where, (tk * tk).reshape(B, H, N * 7, D))
        rv.scatter_add_(2, where, (tv * tv).reshape(B, H, N * 7, D))
    return rk.sqrt(), rv.sqrt()


def assert_slot_grad_close(got, ref, rho, dtype, tol, name):
    """|got - ref| <= atol + rtol * |ref| + 2 * u * rho elementwise; reports the worst ratio."""
    bound = tol["atol"] + tol["rtol"] * ref.abs() + 2.0 * UNIT_ROUNDOFF[dtype] * rho
    err = (got - ref).abs()
    ratio = (err / bound).max().item()
    plain = int((err > tol["atol"] + tol["rtol"] * ref.abs()).sum())
    print(f"{name}: max |err| {err.max().item():.3e}, worst err/bound {ratio:.3f}, "
          f"{plain} entries beyond atol + rtol*|ref| alone")
    assert ratio <= 1.0, f"{name}: error beyond the stated bound (worst ratio {ratio:.3f})"


def protocol_b(q, sk, sv, rounds, causal, res, go=None, gw=None, pairs=None, tol=TOL16):
    """GPU-led: the oracle follows the GPU's picks; every row and gradient compared.
    ``pairs``: (batch, head) pairs of the GPU run that the oracle covers (None: all)."""
    def sub(t):
        if pairs is None:
            return t
        return torch.stack([t[b, h] for b, h in pairs]).unsqueeze(0)
    need_grad = go is not None
    qf, skf, svf = (sub(t).float().clone().requires_grad_(need_grad) for t in (q, sk, sv))
    forced = [sub(i) for i in res["per_round"]]
    out, w, info = oracle.slot_murmurate_forced(qf, skf, svf, forced, causal=causal)
    for r in range(rounds):
        check_indices(forced[r], info["own_idx"][r], info["top8"][r], f"B round {r}")
    torch.testing.assert_close(sub(res["out"]), out.detach(), **tol, msg=lambda m: f"out: {m}")
    torch.testing.assert_close(sub(res["w"]), w.detach(), **tol, msg=lambda m: f"weights: {m}")
    if need_grad:
        ((out * sub(go).float()).sum() + (w * sub(gw)).sum()).backward()
        torch.testing.assert_close(sub(res["grad_q"]), qf.grad, **tol, msg=lambda m: f"grad_q: {m}")
        rk, rv = slot_grad_rho(sub(q), sub(go), forced, info, skf.shape[2])
        assert_slot_grad_close(sub(res["grad_sk"]), skf.grad, rk, q.dtype, tol, "grad_sk")
        assert_slot_grad_close(sub(res["grad_sv"]), svf.grad, rv, q.dtype, tol, "grad_sv")


