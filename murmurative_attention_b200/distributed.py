"""Multi-GPU plumbing for slot_murmurate (one process per GPU, torch.distributed).

The operation shards by (batch, head) pair with no exchange: every pair's
rounds read and write only its own slot table. ``pair_range`` splits the B*H
pairs of a global problem contiguously over ranks; ``local_pairs`` cuts a
rank's share out of a [B, H, ...] tensor as a [1, P_rank, ...] view-compatible
tensor. The MurmurativeAttention training step is data
parallel over the batch: ``allreduce_gradients`` sums the parameter gradients
of all ranks in one flat bucket (NCCL over NVLink on GPUs, gloo on CPUs) and
divides by the world size, like DDP's default averaging.
"""
from __future__ import annotations

from typing import Iterable, Optional, Tuple

import torch
import torch.distributed as dist


def pair_range(total_pairs: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) of the (batch, head) pairs owned by ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total_pairs, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def local_pairs(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's pairs of a [B, H, ...] tensor, as [1, P_rank, ...]."""
    B, H = x.shape[:2]
    s, e = pair_range(B * H, world, rank)
    return x.reshape(1, B * H, *x.shape[2:])[:, s:e]


def gather_pairs(local: torch.Tensor, B: int, H: int, group=None) -> torch.Tensor:
    """Inverse of ``local_pairs``: all ranks' [1, P_r, ...] pieces -> [B, H, ...]."""
    world = dist.get_world_size(group)
    sizes = [pair_range(B * H, world, r) for r in range(world)]
    width = max(e - s for s, e in sizes)
    pad = torch.zeros((1, width) + tuple(local.shape[2:]), dtype=local.dtype, device=local.device)
    pad[:, :local.shape[1]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    full = torch.cat([p[:, :e - s] for p, (s, e) in zip(parts, sizes)], dim=1)
    return full.reshape(B, H, *local.shape[2:])


def allreduce_gradients(params: Iterable[torch.nn.Parameter], group=None, average: bool = True,
                        bucket: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sum (or average) the .grad of ``params`` over the group in one flat bucket.

    One collective per step: the gradients are packed into a contiguous buffer
    (reused when ``bucket`` is given), all-reduced, and unpacked in place.
    Returns the bucket.
    """
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return bucket
    n = sum(g.numel() for g in grads)
    dtype, device = grads[0].dtype, grads[0].device
    if bucket is None or bucket.numel() < n or bucket.dtype != dtype or bucket.device != device:
        bucket = torch.empty(n, dtype=dtype, device=device)
    off = 0
    for g in grads:
        bucket[off:off + g.numel()].copy_(g.reshape(-1))
        off += g.numel()
    dist.all_reduce(bucket[:n], op=dist.ReduceOp.SUM, group=group)
    if average:
        bucket[:n].div_(dist.get_world_size(group))
    off = 0
    for g in grads:
        g.copy_(bucket[off:off + g.numel()].view_as(g))
        off += g.numel()
    return bucket
