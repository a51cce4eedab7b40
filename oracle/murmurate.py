"""CPU restatement of murmurative attention's slot_murmurate path (TEST ORACLE).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, never by the product package.

Every function restates one function of the reference implementation
(beaglabs/murmurative-attention, file src/murmurative/reference.py, cited as
``reference.py:<lines>``) with the same PyTorch operations, so that on the same
inputs it produces the same floating-point results on the CPU. One deliberate
difference: ``torch.topk`` (reference.py:38) returns equal scores in an
implementation-defined order, so ``slot_select`` defaults to a stable
descending sort, which ranks equal scores by the lowest slot index. The two
agree on every row whose top-8 scores are distinct; the only exact ties in
practice are the ``-inf`` scores of causal rows n < 6 (fewer than 7 visible
slots), where the lowest-index rule picks slots n+1, n+2, ...

The north-star operation ``slot_murmurate(q, slots_k, slots_v, rounds, top_k,
causal) -> (out, indices, weights)`` is the reference round loop
(reference.py:177-189) with token keys = token values = q and a zero residual
stream, so ``out`` is the sum over rounds of the attend outputs, and
``indices``/``weights`` are those of the last round.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

TOP_K = 7          # reference.py:38 hard-codes k=7
EMA_EPS = 1e-8     # reference.py:106-107


# ---------------------------------------------------------------------------
# The four phases
# ---------------------------------------------------------------------------

def slot_scores(query: torch.Tensor, slot_keys: torch.Tensor, mask=None, causal=False,
                position_bias=None, effective_M=None) -> torch.Tensor:
    """Masked selection scores, reference.py:14-36."""
    M = slot_keys.shape[2]
    N = query.shape[2]
    em = min(effective_M if effective_M is not None else M, M)
    scores = torch.einsum("bhnd,bhmd->bhnm", query, slot_keys)          # :19
    if position_bias is not None:                                        # :21-22
        scores = scores + position_bias
    if mask is not None:                                                 # :24-25
        scores = scores.masked_fill(mask == 0, float("-inf"))
    if causal:                                                           # :27-31
        future = (torch.arange(M, device=query.device).view(1, 1, 1, M)
                  > torch.arange(N, device=query.device).view(1, 1, N, 1))
        scores = scores.masked_fill(future, float("-inf"))
    if em < M:                                                           # :34-36
        tail = torch.arange(M, device=query.device).view(1, 1, 1, M) >= em
        scores = scores.masked_fill(tail, float("-inf"))
    return scores


def topk_indices(scores: torch.Tensor, tie_rule: str = "lowest_index") -> torch.Tensor:
    """Top-7 slot indices by descending score (reference.py:38).

    ``tie_rule="lowest_index"`` ranks equal scores by ascending slot index
    (stable sort); ``tie_rule="topk"`` calls torch.topk exactly as the
    reference does (used only to time the reference's own CPU path).
    """
    if scores.shape[-1] < TOP_K:
        raise RuntimeError(f"selected index k out of range: need at least {TOP_K} slots, "
                           f"got {scores.shape[-1]}")
    if tie_rule == "topk":
        _, idx = torch.topk(scores, k=TOP_K, dim=-1, sorted=True)
    elif tie_rule == "lowest_index":
        idx = torch.sort(scores, dim=-1, descending=True, stable=True).indices[..., :TOP_K]
    else:
        raise ValueError(tie_rule)
    return idx.to(torch.int64)


def slot_select(query, slot_keys, mask=None, causal=False, position_bias=None,
                effective_M=None, tie_rule: str = "lowest_index") -> torch.Tensor:
    """reference.py:6-39 (``slot_select_reference``)."""
    return topk_indices(slot_scores(query, slot_keys, mask, causal, position_bias,
                                    effective_M), tie_rule)


def slot_attend(query, slot_keys, slot_values, indices, scale: Optional[float] = None,
                logits_out: Optional[list] = None):
    """reference.py:42-68 (``slot_attend_reference``).

    Gathers the selected keys, recomputes their scores *without* any mask
    (reference.py:61-63), softmaxes them and averages the selected values.
    ``logits_out`` (checker instrumentation): the scaled logits are appended to it, with
    their gradient retained when they require one.
    """
    B, H, N, D = query.shape
    M = slot_keys.shape[2]
    K = indices.shape[-1]
    if scale is None:
        scale = 1.0 / (D ** 0.5)                                          # :53-54
    flat = indices.clamp(0, M - 1).reshape(B, H, N * K, 1).expand(-1, -1, -1, D)  # :56-58
    keys = torch.gather(slot_keys, 2, flat).reshape(B, H, N, K, D)        # :59
    logits = torch.einsum("bhnd,bhnkd->bhnk", query, keys) * scale        # :61
    if logits_out is not None:
        if logits.requires_grad:
            logits.retain_grad()
        logits_out.append(logits)
    w = F.softmax(logits, dim=-1)                                         # :63
    vals = torch.gather(slot_values, 2, flat).reshape(B, H, N, K, D)      # :65
    out = torch.einsum("bhnk,bhnkd->bhnd", w, vals)                       # :66
    return out, w.to(torch.float32)                                       # :68


def slot_update(token_keys, token_values, slot_keys, slot_values, indices, weights,
                alpha: float = 0.9):
    """reference.py:71-115 (``slot_update_reference``): fp32 scatter-add then EMA."""
    B, H, N, D = token_keys.shape
    M = slot_keys.shape[2]
    K = indices.shape[-1]
    safe = indices.clamp(0, M - 1)                                        # :84
    dev = token_keys.device
    ksum = torch.zeros(B, H, M, D, device=dev, dtype=torch.float32)       # :87-89
    vsum = torch.zeros(B, H, M, D, device=dev, dtype=torch.float32)
    wsum = torch.zeros(B, H, M, 1, device=dev, dtype=torch.float32)
    for j in range(K):                                                    # :93-103
        col = safe[..., j]
        wj = weights[..., j].unsqueeze(-1).float()
        where = col.unsqueeze(-1)
        ksum.scatter_add_(2, where.expand(-1, -1, -1, D), token_keys.float() * wj)
        vsum.scatter_add_(2, where.expand(-1, -1, -1, D), token_values.float() * wj)
        wsum.scatter_add_(2, where, wj)
    hit = (wsum.squeeze(-1) > 0).unsqueeze(-1)                            # :105, :109
    ku = ksum / (wsum + EMA_EPS)                                          # :106
    vu = vsum / (wsum + EMA_EPS)                                          # :107
    skf = slot_keys.float()
    svf = slot_values.float()
    nk = torch.where(hit, alpha * skf + (1.0 - alpha) * ku, skf)          # :112
    nv = torch.where(hit, alpha * svf + (1.0 - alpha) * vu, svf)          # :113
    return nk.type_as(slot_keys), nv.type_as(slot_values)                 # :115


def slot_diffusion(slot_keys, slot_values, gamma: float = 0.1):
    """reference.py:118-135 (``slot_diffusion_reference``): one Jacobi step of
    the 3-point Laplacian on interior slots; slots 0 and M-1 are fixed."""
    M = slot_keys.shape[2]
    sk = slot_keys.clone()
    sv = slot_values.clone()
    sk[:, :, 1:M - 1] += gamma * (sk[:, :, 0:M - 2] + sk[:, :, 2:M] - 2 * sk[:, :, 1:M - 1])
    sv[:, :, 1:M - 1] += gamma * (sv[:, :, 0:M - 2] + sv[:, :, 2:M] - 2 * sv[:, :, 1:M - 1])
    return sk, sv


# ---------------------------------------------------------------------------
# The north-star composition
# ---------------------------------------------------------------------------

def _check_topk(top_k: int) -> None:
    if top_k != TOP_K:
        raise ValueError(f"top_k must be {TOP_K} (the reference hard-codes k=7), got {top_k}")


def slot_murmurate(q, slots_k, slots_v, rounds: int = 3, top_k: int = 7, causal: bool = False,
                   alpha: float = 0.9, gamma: float = 0.15, scale: Optional[float] = None,
                   tie_rule: str = "lowest_index"):
    """Round loop of reference.py:177-189 with tk = tv = q and x = 0.

    Inputs are upcast to fp32 (the reference computes the update in fp32,
    reference.py:86-115). Returns (out, indices, weights) of the last round.
    Differentiable with respect to q, slots_k and slots_v through autograd.
    """
    _check_topk(top_k)
    qf = q.float()
    sk = slots_k.float()
    sv = slots_v.float()
    out = torch.zeros_like(qf)
    idx = w = None
    for _ in range(rounds):
        idx = slot_select(qf, sk, causal=causal, tie_rule=tie_rule)
        o, w = slot_attend(qf, sk, sv, idx, scale)
        out = out + o                                                     # :187
        sk, sv = slot_update(qf, qf, sk, sv, idx, w, alpha)               # :188
        sk, sv = slot_diffusion(sk, sv, gamma)                            # :189
    if rounds == 0:
        B, H, N, _ = q.shape
        idx = torch.zeros(B, H, N, TOP_K, dtype=torch.int64)
        w = torch.zeros(B, H, N, TOP_K, dtype=torch.float32)
    return out, idx, w


def slot_murmurate_full(x, q_proj, k_proj, v_proj, slot_k_emb, slot_v_emb, num_heads: int = 8,
                        rounds: int = 3, alpha: float = 0.9, gamma: float = 0.15, causal: bool = False,
                        mask=None, position_bias_fn=None, use_dynamic_m: bool = False,
                        slot_ratio: int = 8, tie_rule: str = "lowest_index"):
    """reference.py:138-191 (``slot_murmurate_reference``), the full op: separate token
    keys and values, the residual stream x, an optional selection mask and position
    bias (recomputed from the current x every round), and dynamic M. Inputs are used in
    their own dtype, as the reference does; differentiable through autograd."""
    B, N, D = x.shape
    H = num_heads
    if D % H != 0:                                                        # :157-160
        raise ValueError(f"Embedding dimension D ({D}) must be divisible by num_heads ({H})")
    Dh = D // H
    x_h = x.view(B, N, H, Dh).permute(0, 2, 1, 3)                          # :163-166
    q_h = q_proj.view(B, N, H, Dh).permute(0, 2, 1, 3)
    k_h = k_proj.view(B, N, H, Dh).permute(0, 2, 1, 3)
    v_h = v_proj.view(B, N, H, Dh).permute(0, 2, 1, 3)
    M = slot_k_emb.shape[1]
    slot_k = slot_k_emb.unsqueeze(0).expand(B, -1, -1, -1).contiguous()     # :169-170
    slot_v = slot_v_emb.unsqueeze(0).expand(B, -1, -1, -1).contiguous()
    effective_M = None
    if use_dynamic_m:                                                      # :173-175
        effective_M = min(M, max(32, (N + slot_ratio - 1) // slot_ratio))
    for _ in range(rounds):                                                # :177-189
        pos_bias = position_bias_fn(x_h) if position_bias_fn is not None else None
        indices = slot_select(q_h, slot_k, mask=mask, causal=causal, position_bias=pos_bias,
                              effective_M=effective_M, tie_rule=tie_rule)
        attn_out, attn_w = slot_attend(q_h, slot_k, slot_v, indices)
        x_h = x_h + attn_out
        slot_k, slot_v = slot_update(k_h, v_h, slot_k, slot_v, indices, attn_w, alpha)
        slot_k, slot_v = slot_diffusion(slot_k, slot_v, gamma)
    return x_h.permute(0, 2, 1, 3).contiguous().view(B, N, D)              # :191


def slot_murmurate_forced(q, slots_k, slots_v, forced, causal: bool = False, alpha: float = 0.9,
                          gamma: float = 0.15, scale: Optional[float] = None):
    """The round loop of ``slot_murmurate`` with each round's selection given.

    ``forced[r]`` (int64 [B,H,N,7]) replaces round r's top-7 (reference.py:185): the attend,
    the update and the diffusion of that round use those indices, exactly as
    reference.py:186-189 would use its own. This lets the oracle follow the discrete choices of
    an implementation under test, so that every row's output, weights and gradients can be
    compared even where a near tie made the two pick different slots. The oracle's own choice
    is still computed on its state every round and returned for the index check.

    Returns ``(out, weights_of_last_round, info)``; differentiable with respect to q, slots_k
    and slots_v. ``info["own_idx"][r]`` is the oracle's own top-7 (lowest-index tie rule) on the
    state entering round r, ``info["top8"][r]`` the 8 largest masked scores of each row,
    ``info["w"][r]`` round r's softmax weights and ``info["logits"][r]`` its scaled logits (whose
    ``.grad`` after a backward pass is the softmax adjoint of that round).
    """
    qf = q.float()
    B, H = q.shape[:2]
    sk = slots_k.float().expand(B, H, -1, -1)
    sv = slots_v.float().expand(B, H, -1, -1)
    M = sk.shape[2]
    out = torch.zeros_like(qf)
    info: Dict[str, List[torch.Tensor]] = {"own_idx": [], "top8": [], "w": [], "logits": []}
    w = None
    for idx in forced:
        with torch.no_grad():
            scores = slot_scores(qf.detach(), sk.detach(), causal=causal)             # :14-36
            srt = torch.sort(scores, dim=-1, descending=True, stable=True).values
            info["top8"].append(srt[..., :min(8, M)])
            info["own_idx"].append(topk_indices(scores))                              # :38
            del scores, srt
        o, w = slot_attend(qf, sk, sv, idx.to(torch.int64), scale, info["logits"])    # :186
        info["w"].append(w)
        out = out + o                                                                 # :187
        sk, sv = slot_update(qf, qf, sk, sv, idx.to(torch.int64), w, alpha)          # :188
        sk, sv = slot_diffusion(sk, sv, gamma)                                        # :189
    if w is None:
        w = torch.zeros(B, H, q.shape[2], TOP_K, dtype=torch.float32)
    return out, w, info


@torch.no_grad()
def slot_murmurate_trace(q, slots_k, slots_v, rounds: int = 3, causal: bool = False,
                         alpha: float = 0.9, gamma: float = 0.15,
                         scale: Optional[float] = None) -> Dict[str, object]:
    """Forward pass that also records every round's state.

    Per round r: K[r], V[r] (slot state entering the round), idx[r], w[r],
    top8[r] (the 8 largest masked scores per row, descending), W[r] (per-slot
    weight sums), U[r] (per-slot weighted token means, ksum/(wsum+eps)).
    """
    qf = q.float()
    sk = slots_k.float().expand(q.shape[0], q.shape[1], -1, -1).contiguous()
    sv = slots_v.float().expand(q.shape[0], q.shape[1], -1, -1).contiguous()
    M = sk.shape[2]
    D = q.shape[-1]
    sc = scale if scale is not None else 1.0 / math.sqrt(D)
    out = torch.zeros_like(qf)
    rec: Dict[str, List[torch.Tensor]] = {k: [] for k in ("K", "V", "idx", "w", "top8", "W", "U")}
    for _ in range(rounds):
        rec["K"].append(sk.clone())
        rec["V"].append(sv.clone())
        scores = slot_scores(qf, sk, causal=causal)
        idx = topk_indices(scores)
        rec["top8"].append(torch.sort(scores, dim=-1, descending=True, stable=True)
                           .values[..., :min(8, M)])
        o, w = slot_attend(qf, sk, sv, idx, sc)
        out = out + o
        # weight sums / means exactly as slot_update computes them
        wsum = torch.zeros(*sk.shape[:3], 1)
        ksum = torch.zeros_like(sk)
        for j in range(TOP_K):
            col = idx[..., j].unsqueeze(-1)
            wj = w[..., j].unsqueeze(-1)
            ksum.scatter_add_(2, col.expand(-1, -1, -1, D), qf * wj)
            wsum.scatter_add_(2, col, wj)
        rec["W"].append(wsum.squeeze(-1))
        rec["U"].append(ksum / (wsum + EMA_EPS))
        rec["idx"].append(idx)
        rec["w"].append(w)
        sk, sv = slot_update(qf, qf, sk, sv, idx, w, alpha)
        sk, sv = slot_diffusion(sk, sv, gamma)
    return {"out": out, "K_final": sk, "V_final": sv, **rec}


def _diffuse_transpose(g: torch.Tensor, gamma: float) -> torch.Tensor:
    """Adjoint of slot_diffusion's linear map on one state tensor [..., M, D]."""
    M = g.shape[-2]
    inner = torch.zeros(M, dtype=torch.bool)
    inner[1:M - 1] = True
    diag = torch.where(inner, 1.0 - 2.0 * gamma, 1.0).view(M, 1)
    res = g * diag
    gi = torch.where(inner.view(M, 1), g, torch.zeros_like(g))   # rows that spread to neighbours
    res[..., 1:, :] += gamma * gi[..., :-1, :]
    res[..., :-1, :] += gamma * gi[..., 1:, :]
    return res


@torch.no_grad()
def slot_murmurate_backward_explicit(q, slots_k, slots_v, grad_out, grad_weights=None,
                                     rounds: int = 3, causal: bool = False, alpha: float = 0.9,
                                     gamma: float = 0.15, scale: Optional[float] = None):
    """Hand-derived backward of ``slot_murmurate`` (the math the CUDA kernels use).

    Checked against autograd of ``slot_murmurate`` in tests/test_oracle.py.
    Returns (grad_q, grad_slots_k, grad_slots_v) in fp32.
    """
    tr = slot_murmurate_trace(q, slots_k, slots_v, rounds, causal, alpha, gamma, scale)
    qf = q.float()
    G = grad_out.float()
    B, H, N, D = q.shape
    M = tr["K"][0].shape[2] if rounds else slots_k.shape[2]
    sc = scale if scale is not None else 1.0 / math.sqrt(D)
    dq = torch.zeros_like(qf)
    dK = torch.zeros(B, H, M, D)
    dV = torch.zeros(B, H, M, D)

    def gather(t, idx):
        return torch.gather(t, 2, idx.reshape(B, H, N * TOP_K, 1).expand(-1, -1, -1, t.shape[-1])
                            ).reshape(B, H, N, TOP_K, t.shape[-1])

    def scatter(vals, idx):
        acc = torch.zeros(B, H, M, vals.shape[-1])
        acc.scatter_add_(2, idx.reshape(B, H, N * TOP_K, 1).expand(-1, -1, -1, vals.shape[-1]),
                         vals.reshape(B, H, N * TOP_K, -1))
        return acc

    for r in reversed(range(rounds)):
        K, V, idx, w, W, U = (tr[k][r] for k in ("K", "V", "idx", "w", "W", "U"))
        dKp = _diffuse_transpose(dK, gamma)
        dVp = _diffuse_transpose(dV, gamma)
        hit = (W > 0).unsqueeze(-1)
        dU = torch.where(hit, (1.0 - alpha) * (dKp + dVp), torch.zeros_like(dKp))
        dS = dU / (W.unsqueeze(-1) + EMA_EPS)
        dWs = -(dU * U).sum(-1) / (W + EMA_EPS)
        Kg, Vg, dSg = gather(K, idx), gather(V, idx), gather(dS, idx)
        dWg = torch.gather(dWs, 2, idx.reshape(B, H, N * TOP_K)).reshape(B, H, N, TOP_K)
        dw = (torch.einsum("bhnd,bhnkd->bhnk", G, Vg) + torch.einsum("bhnd,bhnkd->bhnk", qf, dSg)
              + dWg)
        if r == rounds - 1 and grad_weights is not None:
            dw = dw + grad_weights.float()
        da = w * (dw - (w * dw).sum(-1, keepdim=True))
        dq += torch.einsum("bhnk,bhnkd->bhnd", w, dSg) + sc * torch.einsum("bhnk,bhnkd->bhnd", da, Kg)
        dK = torch.where(hit, alpha * dKp, dKp) + scatter((sc * da).unsqueeze(-1) * qf.unsqueeze(-2), idx)
        dV = torch.where(hit, alpha * dVp, dVp) + scatter(w.unsqueeze(-1) * G.unsqueeze(-2), idx)
    return dq, dK, dV


# ---------------------------------------------------------------------------
# Parity helpers
# ---------------------------------------------------------------------------

def row_gap_ok(top8: torch.Tensor, rel: float = 1e-5) -> torch.Tensor:
    """True for rows whose top-7 ranking is numerically unambiguous.

    ``top8`` holds each row's 8 largest masked scores in descending order. A
    row is unambiguous when every adjacent gap among them exceeds
    ``rel * max|finite score|``; pairs of equal ``-inf`` scores (causal rows
    with fewer than 7 visible slots) are resolved by the lowest-index rule and
    do not count as ambiguous.
    """
    fin = torch.isfinite(top8)
    mag = torch.where(fin, top8.abs(), torch.zeros_like(top8)).amax(-1, keepdim=True).clamp_min(1e-30)
    a, b = top8[..., :-1], top8[..., 1:]
    both_inf = (~torch.isfinite(a)) & (~torch.isfinite(b))
    gap = torch.where(torch.isfinite(a) & torch.isfinite(b), a - b,
                      torch.full_like(a, float("inf")))
    ok = (gap > rel * mag) | both_inf
    return ok.all(-1)


# ---------------------------------------------------------------------------
# Seeded inputs for the BASELINE configurations
# ---------------------------------------------------------------------------

CONFIGS = {
    # name: (B, H, N, D, M, dtype, causal, sk_std, sv_std, backward)
    "config1": (2, 4, 128, 64, 256, torch.float32, False, 1.0, 0.0, True),
    "config2": (1, 16, 8192, 64, 256, torch.float16, False, 1.0, 0.0, False),
    "northstar": (1, 16, 8192, 64, 256, torch.float16, False, 1.0, 0.0, True),
    "config3": (8, 16, 4096, 64, 256, torch.bfloat16, True, 1.0 / 8.0, 0.02, True),
    "config5": (4, 32, 65536, 64, 256, torch.bfloat16, True, 1.0, 0.0, True),
}


def make_inputs(name: str = "config1", seed: int = 0, device="cpu", batch=None, heads=None,
                tokens=None):
    """Seeded synthetic inputs with a BASELINE configuration's shapes and
    distributions: q ~ N(0,1); slots_k ~ N(0, sk_std^2); slots_v ~ N(0, sv_std^2)
    (zeros when sv_std == 0); grad_out ~ N(0,1). Drawn in fp32 from one
    torch.Generator on ``device`` in that order, then cast to the config dtype.
    ``batch``/``heads``/``tokens`` override the shape (for bounded samples).
    """
    B, H, N, D, M, dt, causal, sks, svs, _ = CONFIGS[name]
    B = batch or B
    H = heads or H
    N = tokens or N
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g, device=device)
    sk = torch.randn(B, H, M, D, generator=g, device=device) * sks
    sv = (torch.randn(B, H, M, D, generator=g, device=device) * svs if svs > 0
          else torch.zeros(B, H, M, D, device=device))
    go = torch.randn(B, H, N, D, generator=g, device=device)
    return dict(q=q.to(dt), slots_k=sk.to(dt), slots_v=sv.to(dt), grad_out=go.to(dt),
                causal=causal)


def slot_murmurate_layer_reference(x, w_q, w_o, slot_embeddings, heads: int, rounds: int = 3,
                                   causal: bool = False):
    """README.md:82-102 ``MurmurativeAttention.forward`` over the oracle op (fp32)."""
    B, N, Dm = x.shape
    Dh = Dm // heads
    q = (x.float() @ w_q.float().t()).view(B, N, heads, Dh).transpose(1, 2)
    sk = slot_embeddings.float().unsqueeze(0).expand(B, -1, -1, -1)
    sv = torch.zeros_like(sk)
    o, _, _ = slot_murmurate(q, sk, sv, rounds=rounds, causal=causal)
    o = o.transpose(1, 2).reshape(B, N, Dm)
    return o @ w_o.float().t()
