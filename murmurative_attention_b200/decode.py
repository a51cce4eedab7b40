"""Streaming decode over a resident slot pool (the reference's decode plan,
docs/murmurative-attention-kernel-plan.md:154-173; the reference ships no code for it).

After a prefill (``functional.slot_murmurate(..., return_slots=True)`` over the prompt,
or fresh slot embeddings), every new token costs O(M * head_dim) per head, with no
growing cache: select its 7 slots (slots above its absolute position masked when
causal), attend, add to the residual, update the 7 slots with the token's key and value
and diffuse the pool. ``SlotPool.step`` runs all of that as one kernel launch
(``murm_decode_step``) and updates the pool in place. Inference only (no autograd).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .functional import _DT, _dtype_code, _ptr, _stream


def _heads(t: torch.Tensor, H: int, dtype) -> torch.Tensor:
    """[B, H, d] view (from [B, H, d] or [B, H*d]) with unit inner stride in ``dtype``."""
    if t.dim() == 2:
        t = t.view(t.shape[0], H, -1)
    if t.dtype != dtype:
        t = t.to(dtype)
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


class SlotPool:
    """Slot tables of B sequences x H heads, [B, H, M, d], advanced one token at a time."""

    def __init__(self, slot_keys: torch.Tensor, slot_values: torch.Tensor,
                 positions: Optional[torch.Tensor] = None):
        _dtype_code(slot_keys, "slot_keys")
        self.keys = slot_keys.detach().clone().contiguous()
        self.values = slot_values.detach().to(slot_keys.dtype).clone().contiguous()
        B = self.keys.shape[0]
        if positions is None:
            positions = torch.zeros(B, dtype=torch.int64)
        self.positions = positions.to(device=self.keys.device, dtype=torch.int64).clone()

    @classmethod
    def from_embeddings(cls, slot_k_emb: torch.Tensor, slot_v_emb: torch.Tensor, batch: int) -> "SlotPool":
        """Fresh pools from per-head slot embeddings [H, M, d] (reset per sequence)."""
        return cls(slot_k_emb.unsqueeze(0).expand(batch, -1, -1, -1), slot_v_emb.unsqueeze(0).expand(batch, -1, -1, -1))

    @torch.no_grad()
    def step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, x: Optional[torch.Tensor] = None,
             causal: bool = True, alpha: float = 0.9, gamma: float = 0.1, scale: Optional[float] = None,
             return_selection: bool = False):
        """One token per sequence: q, k, v (and the residual x) as [B, H, d] or [B, H*d].
        Returns x + attend in the input's layout (and (indices, weights) [B, H, 7] if
        ``return_selection``); the pool and the positions advance in place."""
        B, H, M, D = self.keys.shape
        dt = self.keys.dtype
        flat = q.dim() == 2
        qh, kh, vh = (_heads(t, H, dt) for t in (q, k, v))
        xh = _heads(x, H, dt) if x is not None else None
        out = torch.empty(B, H, D, device=self.keys.device, dtype=dt)
        idx = torch.empty(B, H, 7, device=out.device, dtype=torch.int64) if return_selection else None
        w = torch.empty(B, H, 7, device=out.device, dtype=torch.float32) if return_selection else None
        s2 = lambda t: _lib.Strides2(t.stride(0), t.stride(1))
        a = _lib.DecodeArgs(
            batch=B, heads=H, slots=M, head_dim=D, dtype=_DT[dt], causal=int(bool(causal)),
            positions=_ptr(self.positions), alpha=float(alpha), gamma=float(gamma),
            scale=float(scale) if scale is not None else 0.0,
            q=_ptr(qh), q_stride=s2(qh), k=_ptr(kh), k_stride=s2(kh), v=_ptr(vh), v_stride=s2(vh),
            x=_ptr(xh), x_stride=s2(xh) if xh is not None else _lib.Strides2(), out=_ptr(out), out_stride=s2(out),
            slot_keys=_ptr(self.keys), sk_stride=_lib.Strides(*self.keys.stride()[:3]),
            slot_values=_ptr(self.values), sv_stride=_lib.Strides(*self.values.stride()[:3]),
            indices=_ptr(idx), weights=_ptr(w))
        _lib.check(_lib.load_library().murm_decode_step(ctypes.byref(a), _stream()))
        self.positions += 1
        res = out.view(B, H * D) if flat else out
        return (res, idx, w) if return_selection else res
