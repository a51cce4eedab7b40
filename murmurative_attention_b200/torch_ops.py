"""``torch.ops.murmurative_attention``: the reference's op namespace over this library.

The reference registers seven operator schemas in the namespace ``murmurative_attention``
(torch-ext/torch_binding.cpp:6-33) with CUDA kernels (:35-43), and its Python layer fetches
them as ``torch.ops.murmurative_attention`` (src/murmurative/ops.py:30-38). Importing this
module defines the same seven schemas, with the same names, argument names and results, and
implements them for CUDA tensors on the per-phase C ABI (murm_ops.cu, through
``functional``): callers of the reference's ops find them here unchanged.

    slot_select_attend, slot_select_attend_backward, slot_update (in place),
    slot_update_backward, slot_diffusion (in place), slot_diffusion_backward,
    slot_update_diffuse (in place)

It also defines the north-star operation of this library as an operator with autograd:

    slot_murmurate(Tensor q, Tensor slots_k, Tensor slots_v, int rounds=3, int top_k=7,
                   bool causal=False, float alpha=0.9, float gamma=0.15, float? scale=None)
        -> (Tensor out, Tensor indices, Tensor weights)

built from ``slot_murmurate_fwd`` (which also returns the block the backward reads) and
``slot_murmurate_bwd``, both on the fused tensor-core C ABI. Every operator has a fake
(meta) implementation, so FakeTensor tracing and ``torch.compile(fullgraph=True)`` see
through them; the sizes the fakes need come from the library's host-only size functions.
There is no CPU kernel: like the reference's ops, these run on CUDA tensors only.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from . import _lib, functional, ops

NS = "murmurative_attention"

# The reference's schemas (torch-ext/torch_binding.cpp:7-32), verbatim: an interface.
REFERENCE_SCHEMAS = {
    "slot_select_attend": "slot_select_attend(Tensor query, Tensor slot_keys, Tensor slot_values, "
                          "Tensor? mask, bool causal, Tensor? position_bias, float? scale, int effective_M) -> "
                          "(Tensor, Tensor, Tensor)",
    "slot_select_attend_backward": "slot_select_attend_backward(Tensor grad_output, Tensor grad_weights, "
                                   "Tensor query, Tensor slot_keys, Tensor slot_values, Tensor indices, "
                                   "Tensor weights, float? scale) -> (Tensor, Tensor, Tensor)",
    "slot_update": "slot_update(Tensor(a!) slot_keys, Tensor(b!) slot_values, Tensor token_keys, "
                   "Tensor token_values, Tensor indices, Tensor weights, float alpha) -> ()",
    "slot_update_backward": "slot_update_backward(Tensor grad_new_sk, Tensor grad_new_sv, Tensor token_keys, "
                            "Tensor token_values, Tensor indices, Tensor weights, float alpha) -> "
                            "(Tensor, Tensor, Tensor, Tensor, Tensor)",
    "slot_diffusion": "slot_diffusion(Tensor(a!) slot_keys, Tensor(b!) slot_values, float gamma) -> ()",
    "slot_diffusion_backward": "slot_diffusion_backward(Tensor grad_new_keys, Tensor grad_new_values, "
                               "float gamma) -> (Tensor, Tensor)",
    "slot_update_diffuse": "slot_update_diffuse(Tensor(a!) slot_keys, Tensor(b!) slot_values, Tensor token_keys, "
                           "Tensor token_values, Tensor indices, Tensor weights, float alpha, float gamma) -> ()",
}
NORTH_STAR_SCHEMAS = {
    "slot_murmurate_fwd": "slot_murmurate_fwd(Tensor q, Tensor slots_k, Tensor slots_v, int rounds, int top_k, "
                          "bool causal, float alpha, float gamma, float? scale) -> "
                          "(Tensor, Tensor, Tensor, Tensor)",
    "slot_murmurate_bwd": "slot_murmurate_bwd(Tensor? grad_out, Tensor? grad_weights, Tensor q, Tensor saved, "
                          "int slots, int rounds, int top_k, bool causal, float alpha, float gamma, "
                          "float? scale) -> (Tensor, Tensor, Tensor)",
    "slot_murmurate": "slot_murmurate(Tensor q, Tensor slots_k, Tensor slots_v, int rounds=3, int top_k=7, "
                      "bool causal=False, float alpha=0.9, float gamma=0.15, float? scale=None) -> "
                      "(Tensor, Tensor, Tensor)",
}

_LIB = torch.library.Library(NS, "DEF")
for _schema in list(REFERENCE_SCHEMAS.values()) + list(NORTH_STAR_SCHEMAS.values()):
    _LIB.define(_schema)


def _q(name: str) -> str:
    return f"{NS}::{name}"


# ---------------------------------------------------------------------------
# The reference's seven operators (CUDA kernels = adapters onto the per-phase C ABI)
# ---------------------------------------------------------------------------
@torch.library.impl(_q("slot_select_attend"), "CUDA", lib=_LIB)
def _select_attend_cuda(query, slot_keys, slot_values, mask, causal, position_bias, scale, effective_M):
    with torch.no_grad():
        return functional.slot_select_attend(query, slot_keys, slot_values, mask, causal, position_bias, scale,
                                             effective_M)


@torch.library.register_fake(_q("slot_select_attend"), lib=_LIB)
def _select_attend_fake(query, slot_keys, slot_values, mask, causal, position_bias, scale, effective_M):
    B, H, N, D = query.shape
    return (query.new_empty(B, H, N, D), query.new_empty(B, H, N, 7, dtype=torch.float32),
            query.new_empty(B, H, N, 7, dtype=torch.int64))


@torch.library.impl(_q("slot_select_attend_backward"), "CUDA", lib=_LIB)
def _select_attend_bwd_cuda(grad_output, grad_weights, query, slot_keys, slot_values, indices, weights, scale):
    return functional.select_attend_backward(grad_output, grad_weights, query, slot_keys, slot_values, indices,
                                             weights, scale)


@torch.library.register_fake(_q("slot_select_attend_backward"), lib=_LIB)
def _select_attend_bwd_fake(grad_output, grad_weights, query, slot_keys, slot_values, indices, weights, scale):
    B, H, N, D = query.shape
    M = slot_keys.shape[2]
    return query.new_empty(B, H, N, D), query.new_empty(B, H, M, D), query.new_empty(B, H, M, D)


@torch.library.impl(_q("slot_update"), "CUDA", lib=_LIB)
def _update_cuda(slot_keys, slot_values, token_keys, token_values, indices, weights, alpha):
    with torch.no_grad():
        nk, nv = functional.slot_update(token_keys, token_values, slot_keys, slot_values, indices, weights, alpha)
        slot_keys.copy_(nk)
        slot_values.copy_(nv)


@torch.library.register_fake(_q("slot_update"), lib=_LIB)
def _update_fake(slot_keys, slot_values, token_keys, token_values, indices, weights, alpha):
    return None


@torch.library.impl(_q("slot_update_backward"), "CUDA", lib=_LIB)
def _update_bwd_cuda(grad_new_sk, grad_new_sv, token_keys, token_values, indices, weights, alpha):
    return functional.slot_update_backward(grad_new_sk, grad_new_sv, token_keys, token_values, indices, weights,
                                           alpha, grad_new_sk.shape[2])


@torch.library.register_fake(_q("slot_update_backward"), lib=_LIB)
def _update_bwd_fake(grad_new_sk, grad_new_sv, token_keys, token_values, indices, weights, alpha):
    B, H, N, D = token_keys.shape
    M = grad_new_sk.shape[2]
    return (token_keys.new_empty(B, H, N, D), token_keys.new_empty(B, H, N, D), token_keys.new_empty(B, H, M, D),
            token_keys.new_empty(B, H, M, D), token_keys.new_empty(B, H, N, 7, dtype=torch.float32))


@torch.library.impl(_q("slot_diffusion"), "CUDA", lib=_LIB)
def _diffusion_cuda(slot_keys, slot_values, gamma):
    with torch.no_grad():
        nk, nv = functional.slot_diffusion(slot_keys, slot_values, gamma)
        slot_keys.copy_(nk)
        slot_values.copy_(nv)


@torch.library.register_fake(_q("slot_diffusion"), lib=_LIB)
def _diffusion_fake(slot_keys, slot_values, gamma):
    return None


@torch.library.impl(_q("slot_diffusion_backward"), "CUDA", lib=_LIB)
def _diffusion_bwd_cuda(grad_new_keys, grad_new_values, gamma):
    return functional.slot_diffusion_backward(grad_new_keys, grad_new_values, gamma)


@torch.library.register_fake(_q("slot_diffusion_backward"), lib=_LIB)
def _diffusion_bwd_fake(grad_new_keys, grad_new_values, gamma):
    return torch.empty_like(grad_new_keys), torch.empty_like(grad_new_values)


@torch.library.impl(_q("slot_update_diffuse"), "CUDA", lib=_LIB)
def _update_diffuse_cuda(slot_keys, slot_values, token_keys, token_values, indices, weights, alpha, gamma):
    with torch.no_grad():
        nk, nv = functional.slot_update(token_keys, token_values, slot_keys, slot_values, indices, weights, alpha)
        nk, nv = functional.slot_diffusion(nk, nv, gamma)
        slot_keys.copy_(nk)
        slot_values.copy_(nv)


@torch.library.register_fake(_q("slot_update_diffuse"), lib=_LIB)
def _update_diffuse_fake(slot_keys, slot_values, token_keys, token_values, indices, weights, alpha, gamma):
    return None


# ---------------------------------------------------------------------------
# The north-star operator with autograd (fused tensor-core C ABI)
# ---------------------------------------------------------------------------
def _out_layout(q: Tensor) -> Tensor:
    """The output's layout: q's own strides when the C ABI reads and writes them in place (unit
    inner stride, non-negative strides that are multiples of 8 elements), else contiguous."""
    st = q.stride()
    ok = st[-1] == 1 and all(s > 0 and s % 8 == 0 for s in st[:3])
    return torch.empty_strided(q.shape, st, dtype=q.dtype, device=q.device) if ok else \
        torch.empty(q.shape, dtype=q.dtype, device=q.device)


def _shape(q, M, rounds, top_k, causal, alpha, gamma, scale):
    return ops._make_shape(q, M, rounds, top_k, causal, alpha, gamma, scale)


@torch.library.impl(_q("slot_murmurate_fwd"), "CUDA", lib=_LIB)
def _fwd_cuda(q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma, scale):
    if top_k != _lib.TOP_K:
        raise ValueError(f"top_k must be {_lib.TOP_K} (the reference hard-codes k=7), got {top_k}")
    out, idx, w, saved, _ = ops._forward(q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma, scale,
                                         out=_out_layout(q))
    return out, idx, w, saved


@torch.library.register_fake(_q("slot_murmurate_fwd"), lib=_LIB)
def _fwd_fake(q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma, scale):
    B, H, N, D = q.shape
    saved_b, _, _ = ops.slot_murmurate_sizes(_shape(q, slots_k.shape[2], rounds, top_k, causal, alpha, gamma, scale))
    return (_out_layout(q), q.new_empty(B, H, N, 7, dtype=torch.int64), q.new_empty(B, H, N, 7, dtype=torch.float32),
            q.new_empty(saved_b, dtype=torch.uint8))


@torch.library.impl(_q("slot_murmurate_bwd"), "CUDA", lib=_LIB)
def _bwd_cuda(grad_out, grad_weights, q, saved, slots, rounds, top_k, causal, alpha, gamma, scale):
    shape = _shape(q, slots, rounds, top_k, causal, alpha, gamma, scale)
    B, H, _, D = q.shape
    go = grad_out if grad_out is not None else torch.zeros_like(q)
    return ops._backward(q, go, grad_weights, saved, shape, (B, H, slots, D), gq=_out_layout(q))


@torch.library.register_fake(_q("slot_murmurate_bwd"), lib=_LIB)
def _bwd_fake(grad_out, grad_weights, q, saved, slots, rounds, top_k, causal, alpha, gamma, scale):
    B, H, _, D = q.shape
    return _out_layout(q), q.new_empty(B, H, slots, D), q.new_empty(B, H, slots, D)


def _fwd_setup(ctx, inputs, output):
    q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma, scale = inputs
    _, _, _, saved = output
    ctx.save_for_backward(q, saved)
    ctx.args = (slots_k.shape[2], rounds, top_k, causal, alpha, gamma, scale)
    ctx.slot_dtypes = (slots_k.dtype, slots_v.dtype)


def _fwd_backward(ctx, grad_out, grad_idx, grad_w, grad_saved):
    q, saved = ctx.saved_tensors
    gq, gsk, gsv = torch.ops.murmurative_attention.slot_murmurate_bwd(grad_out, grad_w, q, saved, *ctx.args)
    return gq, gsk, gsv, None, None, None, None, None, None


torch.library.register_autograd(_q("slot_murmurate_fwd"), _fwd_backward, setup_context=_fwd_setup, lib=_LIB)


@torch.library.impl(_q("slot_murmurate"), "CompositeImplicitAutograd", lib=_LIB)
def _slot_murmurate(q, slots_k, slots_v, rounds=3, top_k=7, causal=False, alpha=0.9, gamma=0.15, scale=None):
    out, idx, w, _ = torch.ops.murmurative_attention.slot_murmurate_fwd(q, slots_k, slots_v, rounds, top_k, causal,
                                                                         alpha, gamma, scale)
    return out, idx, w


def slot_murmurate(q: Tensor, slots_k: Tensor, slots_v: Tensor, rounds: int = 3, top_k: int = 7,
                   causal: bool = False, *, alpha: float = 0.9, gamma: float = 0.15,
                   scale: Optional[float] = None) -> Tuple[Tensor, Tensor, Tensor]:
    """``torch.ops.murmurative_attention.slot_murmurate``: the same operation and results as
    ``murmurative_attention_b200.slot_murmurate``, as a registered operator (traceable by
    torch.compile)."""
    return torch.ops.murmurative_attention.slot_murmurate(q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma,
                                                          scale)
