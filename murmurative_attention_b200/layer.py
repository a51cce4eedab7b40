"""The ``MurmurativeAttention`` layer of the reference README (README.md:82-102).

q_proj -> slot_murmurate over per-head slot embeddings (slots_v starts at
zero) -> o_proj. The reference ships this module only as README text; here it
is a real module over the B200 op. The head split is a strided view: the op
reads q in the projection's [B, N, H, d] memory and writes its output in the
same layout, so neither transpose copies.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .ops import slot_murmurate
from .torch_ops import slot_murmurate as slot_murmurate_op


class MurmurativeAttention(nn.Module):
    def __init__(self, dim: int = 256, heads: int = 4, slots: int = 256, rounds: int = 3, top_k: int = 7,
                 causal: bool = False, device=None, dtype=None):
        super().__init__()
        if dim % heads:
            raise ValueError(f"Embedding dimension D ({dim}) must be divisible by num_heads ({heads})")
        self.dim, self.heads, self.slots, self.rounds, self.top_k = dim, heads, slots, rounds, top_k
        self.causal = causal
        self.head_dim = dim // heads
        kw = dict(device=device, dtype=dtype)
        self.q_proj = nn.Linear(dim, dim, bias=False, **kw)
        self.o_proj = nn.Linear(dim, dim, bias=False, **kw)
        self.slot_embeddings = nn.Parameter(torch.randn(heads, slots, self.head_dim, **kw))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, N, D = x.shape
        q = self.q_proj(x).view(B, N, self.heads, self.head_dim).transpose(1, 2)
        slots_k = self.slot_embeddings.unsqueeze(0).expand(B, -1, -1, -1)
        slots_v = torch.zeros_like(slots_k)
        # under torch.compile the registered operator (traceable, same kernels); eagerly the
        # autograd Function, which skips the dispatcher's Python round trip
        op = slot_murmurate_op if torch.compiler.is_compiling() else slot_murmurate
        attn_out, _, _ = op(q, slots_k, slots_v, rounds=self.rounds, top_k=self.top_k, causal=self.causal)
        attn_out = attn_out.transpose(1, 2).reshape(B, N, D)
        return self.o_proj(attn_out)
