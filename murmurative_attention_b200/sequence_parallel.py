"""Sequence parallelism for long contexts with few (batch, head) pairs.

One process per GPU; the ranks of ``group`` hold consecutive, equal token shards of the
same sequences (rank r: tokens [r*n, (r+1)*n)) and the full slot tables. Per round each
rank selects and attends its own tokens; the only exchange is one all-reduce of the slot
partial sums (weighted token keys and values and the weight sums, reference.py:87-103),
since sums over token shards add up; the EMA (reference.py:105-115) and the diffusion
(reference.py:118-135) then run replicated on every rank. Gradients flow back through
the all-reduce (its adjoint is another all-reduce). The causal mask uses the global token
positions.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.distributed.nn.functional as dnn

from . import functional as F

EMA_EPS = 1e-8


def slot_murmurate_sp(q: torch.Tensor, slots_k: torch.Tensor, slots_v: torch.Tensor, rounds: int = 3,
                      causal: bool = False, alpha: float = 0.9, gamma: float = 0.15,
                      group: Optional[dist.ProcessGroup] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The north-star op (token keys = token values = q, zero residual) over this rank's
    token shard ``q`` [B, H, n, d]; returns (out, indices, weights) for the shard, equal
    to the corresponding rows of the single-process result."""
    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(group), dist.get_rank(group)
    else:  # no process group: one rank holding every token
        world, rank = 1, 0
    B, H, n, D = q.shape
    M = slots_k.shape[2]
    mask = None
    if causal:  # slot m visible to global token rank*n + i when m <= rank*n + i
        pos = torch.arange(n, device=q.device) + rank * n
        mask = (torch.arange(M, device=q.device).view(1, M) <= pos.view(n, 1)).to(torch.uint8)
    sk, sv = slots_k, slots_v
    out = None
    idx = w = None
    for _ in range(rounds):
        o, w, idx = F.slot_select_attend(q, sk, sv, mask=mask)
        out = o if out is None else out + o
        ks, vs, ws = F.slot_sums(q, q, idx, w, M)
        if world > 1:
            ks = dnn.all_reduce(ks, group=group)
            vs = dnn.all_reduce(vs, group=group)
            ws = dnn.all_reduce(ws, group=group)
        hit = (ws > 0).unsqueeze(-1)
        den = (ws + EMA_EPS).unsqueeze(-1)
        skf, svf = sk.float(), sv.float()
        sk = torch.where(hit, alpha * skf + (1.0 - alpha) * (ks / den), skf).to(slots_k.dtype)
        sv = torch.where(hit, alpha * svf + (1.0 - alpha) * (vs / den), svf).to(slots_v.dtype)
        sk, sv = F.slot_diffusion(sk, sv, gamma)
    return out, idx, w
