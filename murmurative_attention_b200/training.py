"""Data-parallel training step of the ``MurmurativeAttention`` layer.

the layer (q_proj -> slot_murmurate -> o_proj, README.md:82-102)
trained data-parallel, one process per GPU, each rank on its own sequences. The only
exchange is the gradient average of the layer's parameters (q_proj, o_proj and the slot
embeddings) over NCCL. ``GradientAverager`` starts each parameter's all-reduce as soon as
autograd has accumulated its gradient (o_proj's comes first, while the slot op's backward
is still running) and ``finish()`` waits for all of them before the optimizer step, which
is how DDP overlaps communication with the backward pass.
"""
from __future__ import annotations

from typing import Callable, Iterable, List, Optional

import torch
import torch.distributed as dist


class GradientAverager:
    """Asynchronous per-parameter gradient averaging over a process group."""

    def __init__(self, params: Iterable[torch.nn.Parameter], group=None):
        self.group = group
        self.params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self._pending: List = []
        self._hooks = []
        if self.world > 1:
            for p in self.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._launch))

    def _launch(self, p: torch.nn.Parameter) -> None:
        self._pending.append((p, dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=self.group, async_op=True)))

    def finish(self) -> None:
        """Wait for every launched all-reduce and turn the sums into averages."""
        for p, work in self._pending:
            work.wait()
            p.grad.div_(self.world)
        self._pending.clear()

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks.clear()


def mean_square_loss(y: torch.Tensor) -> torch.Tensor:
    return y.float().square().mean()


def dp_train_step(model: torch.nn.Module, x: torch.Tensor, optimizer: torch.optim.Optimizer,
                  averager: Optional[GradientAverager] = None,
                  loss_fn: Callable[[torch.Tensor], torch.Tensor] = mean_square_loss) -> torch.Tensor:
    """One training step: forward, loss, backward (gradients averaged over the group
    while it runs), optimizer step. Returns the detached local loss."""
    optimizer.zero_grad(set_to_none=False)
    loss = loss_fn(model(x))
    loss.backward()
    if averager is not None:
        averager.finish()
    optimizer.step()
    return loss.detach()
