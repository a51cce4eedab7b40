"""PyTorch-facing slot_murmurate: argument handling, buffers, autograd.

Mirrors the reference's Python op layer (src/murmurative/ops.py):
- ``slot_murmurate(q, slots_k, slots_v, rounds=3, top_k=7, causal=False)``
  returns ``(out, indices, weights)`` — the call shape the reference README
  shows (README.md:61-69, 95-102) and BASELINE's north-star names;
- dtype errors raise ``TypeError`` (ops.py:41-48), a missing library or CUDA
  device ``RuntimeError`` (_cuda_kernels.py:19-46), bad shapes
  ``RuntimeError`` (the reference's TORCH_CHECKs);
- gradients flow to q, slots_k and slots_v (ops.py:55-208's autograd
  Functions, here one Function for the whole round loop).

All arithmetic runs in libmurm_b200.so through the C ABI; this module only
allocates tensors, reads strides and the current stream, and calls it.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.MURM_F32, torch.float16: _lib.MURM_F16, torch.bfloat16: _lib.MURM_BF16}


def _dtype_code(t: torch.Tensor, name: str) -> int:
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise TypeError(f"slot_murmurate supports float32, float16 and bfloat16 tensors, but {name} "
                        f"has dtype {t.dtype}")
    return code


def _rows_ok(t: torch.Tensor, allow_batch_broadcast: bool) -> bool:
    st = t.stride()
    if st[-1] != 1 or t.data_ptr() % 16:
        return False
    for i, s in enumerate(st[:3]):
        if s < 0 or (s == 0 and not (i == 0 and allow_batch_broadcast)) or s % 8:
            return False
    return True


def _rows(t: torch.Tensor, allow_batch_broadcast: bool = False) -> torch.Tensor:
    """The tensor itself when the C ABI can read it in place, else a copy."""
    return t if _rows_ok(t, allow_batch_broadcast) else t.contiguous()


def _strides(t: torch.Tensor) -> "_lib.Strides":
    return _lib.Strides(*t.stride()[:3])


def _make_shape(q, M, rounds, top_k, causal, alpha, gamma, scale) -> "_lib.Shape":
    B, H, N, D = q.shape
    return _lib.Shape(B, H, N, M, D, int(rounds), int(top_k), 1 if causal else 0, float(alpha), float(gamma),
                      float(scale) if scale is not None else 0.0, _DTYPES[q.dtype])


def slot_murmurate_sizes(shape: "_lib.Shape") -> Tuple[int, int, int]:
    """(saved_bytes, forward_workspace_bytes, backward_workspace_bytes)."""
    lib = _lib.load_library()
    a, b, c = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(lib.murm_slot_murmurate_sizes(ctypes.byref(shape), ctypes.byref(a), ctypes.byref(b),
                                             ctypes.byref(c)))
    return a.value, b.value, c.value


def _check_inputs(q, slots_k, slots_v):
    for name, t in (("q", q), ("slots_k", slots_k), ("slots_v", slots_v)):
        _dtype_code(t, name)
        if t.dim() != 4:
            raise RuntimeError(f"{name} must be 4-D [B, H, rows, head_dim], got shape {tuple(t.shape)}")
        if not t.is_cuda:
            raise RuntimeError("murmurative CUDA kernels require CUDA tensors; "
                               f"{name} is on {t.device}")
    if slots_k.dtype != q.dtype or slots_v.dtype != q.dtype:
        raise TypeError(f"q, slots_k and slots_v must share a dtype, got {q.dtype}, {slots_k.dtype}, "
                        f"{slots_v.dtype}")
    B, H, N, D = q.shape
    if slots_k.shape != slots_v.shape or slots_k.shape[0] != B or slots_k.shape[1] != H or slots_k.shape[3] != D:
        raise RuntimeError(f"slots_k/slots_v must be [B={B}, H={H}, M, d={D}], got {tuple(slots_k.shape)} and "
                           f"{tuple(slots_v.shape)}")
    if slots_k.device != q.device or slots_v.device != q.device:
        raise RuntimeError("q, slots_k and slots_v must be on the same device")


def _forward(q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma, scale, out=None):
    lib = _lib.load_library()
    _check_inputs(q, slots_k, slots_v)
    if not torch.cuda.is_available():
        raise RuntimeError("murmurative CUDA kernels require a CUDA-capable device, but none is available.")
    q = _rows(q)
    sk = _rows(slots_k, True)
    sv = _rows(slots_v, True)
    B, H, N, D = q.shape
    shape = _make_shape(q, sk.shape[2], rounds, top_k, causal, alpha, gamma, scale)
    saved_b, fws_b, _ = slot_murmurate_sizes(shape)
    dev = q.device
    if out is None or not _rows_ok(out, False):
        out = torch.empty_like(q)  # keeps q's layout, e.g. [B,N,H,d] memory for a transposed view
    if not _rows_ok(out, False):
        out = torch.empty(q.shape, dtype=q.dtype, device=dev)
    idx = torch.empty(B, H, N, _lib.TOP_K, dtype=torch.int64, device=dev)
    w = torch.empty(B, H, N, _lib.TOP_K, dtype=torch.float32, device=dev)
    saved = torch.empty(saved_b, dtype=torch.uint8, device=dev)
    ws = torch.empty(fws_b, dtype=torch.uint8, device=dev)
    args = _lib.FwdArgs(shape, q.data_ptr(), _strides(q), sk.data_ptr(), _strides(sk), sv.data_ptr(),
                        _strides(sv), out.data_ptr(), _strides(out), idx.data_ptr(), w.data_ptr(),
                        saved.data_ptr() or None, saved_b, ws.data_ptr() or None, fws_b)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.murm_slot_murmurate_fwd(ctypes.byref(args), ctypes.c_void_p(stream)))
    return out, idx, w, saved, shape


def _backward(q, grad_out, grad_w, saved, shape, slots_shape, gq=None):
    lib = _lib.load_library()
    q = _rows(q)
    go = _rows(grad_out.to(q.dtype))
    gw = grad_w.float().contiguous() if grad_w is not None else None
    _, _, bws_b = slot_murmurate_sizes(shape)
    dev = q.device
    if gq is None or not _rows_ok(gq, False):
        gq = torch.empty_like(q)
    if not _rows_ok(gq, False):
        gq = torch.empty(q.shape, dtype=q.dtype, device=dev)
    gsk = torch.empty(slots_shape, dtype=q.dtype, device=dev)
    gsv = torch.empty(slots_shape, dtype=q.dtype, device=dev)
    ws = torch.empty(bws_b, dtype=torch.uint8, device=dev)
    args = _lib.BwdArgs(shape, q.data_ptr(), _strides(q), go.data_ptr(), _strides(go),
                        gw.data_ptr() if gw is not None else None, saved.data_ptr() or None, saved.numel(),
                        gq.data_ptr(), _strides(gq), gsk.data_ptr(), _strides(gsk), gsv.data_ptr(),
                        _strides(gsv), ws.data_ptr(), bws_b)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.murm_slot_murmurate_bwd(ctypes.byref(args), ctypes.c_void_p(stream)))
    return gq, gsk, gsv


class _SlotMurmurate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma, scale):
        out, idx, w, saved, shape = _forward(q, slots_k, slots_v, rounds, top_k, causal, alpha, gamma, scale)
        ctx.save_for_backward(q, saved)
        ctx.shape = shape
        ctx.slots_shape = tuple(slots_k.shape)
        ctx.mark_non_differentiable(idx)
        return out, idx, w

    @staticmethod
    def backward(ctx, grad_out, grad_idx, grad_w):
        q, saved = ctx.saved_tensors
        if grad_out is None:
            grad_out = torch.zeros_like(q)
        gq, gsk, gsv = _backward(q, grad_out, grad_w, saved, ctx.shape, ctx.slots_shape)
        return gq, gsk, gsv, None, None, None, None, None, None


def slot_murmurate(q: torch.Tensor, slots_k: torch.Tensor, slots_v: torch.Tensor, rounds: int = 3,
                   top_k: int = 7, causal: bool = False, *, alpha: float = 0.9, gamma: float = 0.15,
                   scale: Optional[float] = None):
    """Murmurative slot attention over R rounds on a B200.

    Args:
        q: [B, H, N, d] queries; also the token keys and values of the slot
           update. fp16, bf16 or fp32; any strides with unit inner stride
           (e.g. the [B, N, H, d] memory of ``x.view(B,N,H,d).transpose(1,2)``).
        slots_k, slots_v: [B, H, M, d] initial slot keys / values (same
           dtype); a batch stride of 0 (``.expand``) is read in place.
        rounds: R >= 0. top_k: must be 7. causal: token n sees slots m <= n.
        alpha, gamma: EMA keep factor and diffusion step (reference defaults
           0.9 and 0.15). scale: logit scale, default 1/sqrt(d).

    Returns:
        out [B, H, N, d] (q's dtype and layout): sum of the R attend outputs;
        indices [B, H, N, 7] int64: last round's slots, by descending score
        (ties to the lower slot index); weights [B, H, N, 7] fp32: last
        round's softmax weights.
    """
    if top_k != _lib.TOP_K:
        raise ValueError(f"top_k must be {_lib.TOP_K} (the reference hard-codes k=7), got {top_k}")
    return _SlotMurmurate.apply(q, slots_k, slots_v, int(rounds), int(top_k), bool(causal), float(alpha),
                                float(gamma), scale)


def slot_murmurate_host_step(q: torch.Tensor, slots_k: torch.Tensor, slots_v: torch.Tensor,
                             grad_out: torch.Tensor, rounds: int = 3, top_k: int = 7, causal: bool = False, *,
                             alpha: float = 0.9, gamma: float = 0.15, scale: Optional[float] = None,
                             groups: int = 0, outputs: Optional[Tuple[torch.Tensor, ...]] = None,
                             device: Optional[torch.device] = None):
    """Forward and backward of :func:`slot_murmurate` for tensors in host memory.

    The drop-in for the reference's CPU path: ``out, idx, w = slot_murmurate(q, slots_k, slots_v)``
    on CPU tensors followed by ``out.backward(grad_out)`` (reference.py:138-191 and its autograd
    backward). q, grad_out [B, H, N, d] and slots_k, slots_v [B, H, M, d] are contiguous CPU
    tensors of one dtype (pinned memory lets the copies overlap the kernels). The (batch, head)
    pairs run in ``groups`` (0: automatic) through a copy-in / compute / copy-out pipeline on the GPU
    (``murm_slot_murmurate_host_step``). Returns CPU tensors
    ``(out, indices, weights, grad_q, grad_slots_k, grad_slots_v)``, written into ``outputs``
    when given (six tensors of those shapes and dtypes); blocks until they are filled.
    """
    lib = _lib.load_library()
    if top_k != _lib.TOP_K:
        raise ValueError(f"top_k must be {_lib.TOP_K} (the reference hard-codes k=7), got {top_k}")
    for name, t in (("q", q), ("slots_k", slots_k), ("slots_v", slots_v), ("grad_out", grad_out)):
        _dtype_code(t, name)
        if t.dim() != 4 or t.is_cuda or not t.is_contiguous():
            raise RuntimeError(f"{name} must be a contiguous 4-D CPU tensor, got shape {tuple(t.shape)} on "
                               f"{t.device}")
        if t.dtype != q.dtype:
            raise TypeError(f"every tensor must have q's dtype {q.dtype}; {name} is {t.dtype}")
    B, H, N, D = q.shape
    if grad_out.shape != q.shape:
        raise RuntimeError(f"grad_out must have q's shape {tuple(q.shape)}, got {tuple(grad_out.shape)}")
    if slots_k.shape != slots_v.shape or tuple(slots_k.shape[:2]) != (B, H) or slots_k.shape[3] != D:
        raise RuntimeError(f"slots_k/slots_v must be [B={B}, H={H}, M, d={D}], got {tuple(slots_k.shape)} and "
                           f"{tuple(slots_v.shape)}")
    if not torch.cuda.is_available():
        raise RuntimeError("murmurative CUDA kernels require a CUDA-capable device, but none is available.")
    M = slots_k.shape[2]
    shape = _make_shape(q, M, rounds, top_k, causal, alpha, gamma, scale)
    if outputs is None:
        pin = q.is_pinned()
        outputs = (torch.empty(q.shape, dtype=q.dtype, pin_memory=pin),
                   torch.empty(B, H, N, _lib.TOP_K, dtype=torch.int64, pin_memory=pin),
                   torch.empty(B, H, N, _lib.TOP_K, dtype=torch.float32, pin_memory=pin),
                   torch.empty(q.shape, dtype=q.dtype, pin_memory=pin),
                   torch.empty(slots_k.shape, dtype=q.dtype, pin_memory=pin),
                   torch.empty(slots_k.shape, dtype=q.dtype, pin_memory=pin))
    out, idx, w, gq, gsk, gsv = outputs
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    nbytes = ctypes.c_size_t()
    _lib.check(lib.murm_host_step_sizes(ctypes.byref(shape), int(groups), ctypes.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=dev)
    args = _lib.HostStepArgs(shape, q.data_ptr(), slots_k.data_ptr(), slots_v.data_ptr(), grad_out.data_ptr(),
                             out.data_ptr(), idx.data_ptr(), w.data_ptr(), gq.data_ptr(), gsk.data_ptr(),
                             gsv.data_ptr(), int(groups), ws.data_ptr(), nbytes.value)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        _lib.check(lib.murm_slot_murmurate_host_step(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream)))
        stream.synchronize()
    return outputs
