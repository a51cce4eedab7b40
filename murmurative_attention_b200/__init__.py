"""B200-native (sm_100a) murmurative slot attention: ``slot_murmurate`` forward and backward.

The compute runs in ``libmurm_b200.so`` (hand-written CUDA for sm_100a behind
the C ABI of include/murm.h); this package is the PyTorch-facing host side.
"""
from .ops import slot_murmurate, slot_murmurate_host_step, slot_murmurate_sizes  # noqa: F401
from .layer import MurmurativeAttention  # noqa: F401
from . import torch_ops  # noqa: F401  (registers torch.ops.murmurative_attention.*)

__version__ = "0.1.0"
__all__ = ["slot_murmurate", "slot_murmurate_host_step", "slot_murmurate_sizes", "MurmurativeAttention"]
