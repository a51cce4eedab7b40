"""The reference's full op surface (src/murmurative/ops.py) over the per-phase C ABI.

Same names, arguments and results as the reference's ``ops`` module:

- ``slot_select_attend(query, slot_keys, slot_values, mask, causal, position_bias, scale,
  effective_M) -> (output, weights, indices)``   (ops.py:246-279)
- ``slot_select(...) -> indices`` and ``slot_attend(query, slot_keys, slot_values, indices,
  scale) -> (output, weights)``                   (ops.py:219-243)
- ``slot_update(token_keys, token_values, slot_keys, slot_values, indices, weights, alpha)
  -> (new_slot_keys, new_slot_values)``           (ops.py:282-308)
- ``slot_diffusion(slot_keys, slot_values, gamma) -> (slot_keys, slot_values)``
                                                   (ops.py:311-327)
- ``slot_murmurate(x, q_proj, k_proj, v_proj, slot_k_emb, slot_v_emb, num_heads, rounds,
  alpha, gamma, causal, mask, position_bias_fn, use_dynamic_m, slot_ratio, ...)
  -> output [B, N, D]``                            (ops.py:330-422)

All of them are differentiable (with respect to the float inputs; indices are not) and
run on the CUDA-core kernels of murm_ops.cu: a selection mask (nonzero = keep, any shape
that broadcasts to [B, H, N, M]), a position bias (broadcasting likewise) that enters the
selection only, dynamic M, separate token keys and values, head_dim a multiple of 8 up to
128 and M up to 1024. fp32, fp16 and bf16 tensors on a CUDA device; other dtypes raise
TypeError, a missing library or a CPU tensor RuntimeError, as the reference does
(ops.py:41-48, _cuda_kernels.py:19-46). For the north-star case (token keys = token values
= q, no residual, mask or bias) ``murmurative_attention_b200.slot_murmurate`` is the
fused tensor-core operation.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional, Tuple

import torch

from . import _lib

_DT = {torch.float32: _lib.MURM_F32, torch.float16: _lib.MURM_F16, torch.bfloat16: _lib.MURM_BF16}


def _dtype_code(t: torch.Tensor, name: str) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"{name} must be float32, float16 or bfloat16, got {t.dtype}")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    return _DT[t.dtype]


def _rows(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """A [B, H, X, d] view with unit inner stride in ``dtype``."""
    if t.dtype != dtype:
        t = t.to(dtype)
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def _s3(t: torch.Tensor):
    return _lib.Strides(t.stride(0), t.stride(1), t.stride(2))


def _s4(t: torch.Tensor):
    return _lib.Strides4(*t.stride())


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _shape(B, H, N, M, D, code):
    return _lib.PhaseShape(batch=B, heads=H, tokens=N, slots=M, head_dim=D, dtype=code)


def _sizes(shape) -> Tuple[int, int]:
    a, b = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(_lib.load_library().murm_phase_sizes(ctypes.byref(shape), ctypes.byref(a), ctypes.byref(b)))
    return a.value, b.value


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _broadcast4(t: Optional[torch.Tensor], B, H, N, M, dtype, device) -> Optional[torch.Tensor]:
    if t is None:
        return None
    t = t.to(device=device, dtype=dtype)
    while t.dim() < 4:
        t = t.unsqueeze(0)
    return t.expand(B, H, N, M)


class _SelectAttend(torch.autograd.Function):
    @staticmethod
    def forward(ctx, query, slot_keys, slot_values, mask, causal, position_bias, scale, effective_M, indices_in):
        lib = _lib.load_library()
        code = _dtype_code(query, "query")
        dt = query.dtype
        q = _rows(query, dt)
        sk = _rows(slot_keys, dt)
        sv = _rows(slot_values, dt)
        B, H, N, D = q.shape
        M = sk.shape[2]
        dev = q.device
        out = torch.empty(B, H, N, D, device=dev, dtype=dt)
        weights = torch.empty(B, H, N, 7, device=dev, dtype=torch.float32)
        indices = torch.empty(B, H, N, 7, device=dev, dtype=torch.int64)
        m4 = _broadcast4(mask != 0 if mask is not None else None, B, H, N, M, torch.uint8, dev)
        b4 = _broadcast4(position_bias, B, H, N, M, dt, dev)
        idx_in = indices_in.to(device=dev, dtype=torch.int64).contiguous() if indices_in is not None else None
        a = _lib.SelectAttendArgs(
            shape=_shape(B, H, N, M, D, code), causal=int(bool(causal)), effective_m=int(effective_M or 0),
            scale=float(scale) if scale is not None else 0.0,
            q=_ptr(q), q_stride=_s3(q), slot_keys=_ptr(sk), sk_stride=_s3(sk), slot_values=_ptr(sv),
            sv_stride=_s3(sv), mask=_ptr(m4), mask_stride=_s4(m4) if m4 is not None else _lib.Strides4(),
            position_bias=_ptr(b4), bias_stride=_s4(b4) if b4 is not None else _lib.Strides4(),
            indices_in=_ptr(idx_in), out=_ptr(out), out_stride=_s3(out), indices=_ptr(indices),
            weights=_ptr(weights))
        _lib.check(lib.murm_select_attend_fwd(ctypes.byref(a), _stream()))
        ctx.save_for_backward(q, sk, sv, indices, weights)
        ctx.scale = scale
        ctx.in_dtypes = (query.dtype, slot_keys.dtype, slot_values.dtype)
        ctx.mark_non_differentiable(indices)
        return out, weights, indices

    @staticmethod
    def backward(ctx, grad_out, grad_weights, _grad_indices):
        q, sk, sv, indices, weights = ctx.saved_tensors
        gq, gsk, gsv = select_attend_backward(grad_out, grad_weights, q, sk, sv, indices, weights, ctx.scale)
        dq_t, dk_t, dv_t = ctx.in_dtypes
        return gq.to(dq_t), gsk.to(dk_t), gsv.to(dv_t), None, None, None, None, None, None


def select_attend_backward(grad_out: Optional[torch.Tensor], grad_weights: Optional[torch.Tensor],
                           query: torch.Tensor, slot_keys: torch.Tensor, slot_values: torch.Tensor,
                           indices: torch.Tensor, weights: torch.Tensor,
                           scale: Optional[float]) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients of slot_select_attend's output and weights with respect to query, slot_keys
    and slot_values (in query's dtype), given the forward's indices and weights: the
    reference's slot_select_attend_backward (torch_binding.cpp:11-14)."""
    lib = _lib.load_library()
    dt = query.dtype
    q = _rows(query, dt)
    sk = _rows(slot_keys, dt)
    sv = _rows(slot_values, dt)
    B, H, N, D = q.shape
    M = sk.shape[2]
    shape = _shape(B, H, N, M, D, _dtype_code(q, "query"))
    _, ws_bytes = _sizes(shape)
    ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
    go = _rows(grad_out if grad_out is not None else torch.zeros_like(q), dt)
    gw = grad_weights.float().contiguous() if grad_weights is not None else None
    idx = indices.to(device=q.device, dtype=torch.int64).contiguous()
    w = weights.to(device=q.device, dtype=torch.float32).contiguous()
    gq = torch.empty(B, H, N, D, device=q.device, dtype=dt)
    gsk = torch.empty(B, H, M, D, device=q.device, dtype=dt)
    gsv = torch.empty(B, H, M, D, device=q.device, dtype=dt)
    a = _lib.SelectAttendBwdArgs(
        shape=shape, scale=float(scale) if scale is not None else 0.0,
        q=_ptr(q), q_stride=_s3(q), slot_keys=_ptr(sk), sk_stride=_s3(sk), slot_values=_ptr(sv),
        sv_stride=_s3(sv), indices=_ptr(idx), weights=_ptr(w), grad_out=_ptr(go),
        go_stride=_s3(go), grad_weights=_ptr(gw), grad_q=_ptr(gq), gq_stride=_s3(gq),
        grad_slot_keys=_ptr(gsk), gsk_stride=_s3(gsk), grad_slot_values=_ptr(gsv), gsv_stride=_s3(gsv),
        workspace=_ptr(ws), workspace_bytes=ws_bytes)
    _lib.check(lib.murm_select_attend_bwd(ctypes.byref(a), _stream()))
    return gq, gsk, gsv


def _update_forward(token_keys, token_values, slot_keys, slot_values, indices, weights, alpha):
    """murm_slot_update_fwd: new slot tables (slot_keys' dtype) and the saved block (per-slot
    means and weight sums, which depend on the tokens, indices and weights only)."""
    lib = _lib.load_library()
    code = _dtype_code(slot_keys, "slot_keys")
    dt = slot_keys.dtype
    tk = _rows(token_keys, dt)
    tv = _rows(token_values, dt)
    sk = _rows(slot_keys, dt)
    sv = _rows(slot_values, dt)
    B, H, N, D = tk.shape
    M = sk.shape[2]
    shape = _shape(B, H, N, M, D, code)
    saved_bytes, ws_bytes = _sizes(shape)
    dev = tk.device
    saved = torch.empty(saved_bytes, device=dev, dtype=torch.uint8)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    idx = indices.to(device=dev, dtype=torch.int64).contiguous()
    w = weights.to(device=dev, dtype=torch.float32).contiguous()
    nk = torch.empty(B, H, M, D, device=dev, dtype=dt)
    nv = torch.empty(B, H, M, D, device=dev, dtype=dt)
    a = _lib.SlotUpdateArgs(
        shape=shape, alpha=float(alpha), token_keys=_ptr(tk), tk_stride=_s3(tk), token_values=_ptr(tv),
        tv_stride=_s3(tv), slot_keys=_ptr(sk), sk_stride=_s3(sk), slot_values=_ptr(sv), sv_stride=_s3(sv),
        indices=_ptr(idx), weights=_ptr(w), new_slot_keys=_ptr(nk), nsk_stride=_s3(nk),
        new_slot_values=_ptr(nv), nsv_stride=_s3(nv), saved=_ptr(saved), saved_bytes=saved_bytes,
        workspace=_ptr(ws), workspace_bytes=ws_bytes)
    _lib.check(lib.murm_slot_update_fwd(ctypes.byref(a), _stream()))
    return nk, nv, saved, (tk, tv, idx, w)


def slot_update_backward(grad_new_keys: Optional[torch.Tensor], grad_new_values: Optional[torch.Tensor],
                         token_keys: torch.Tensor, token_values: torch.Tensor, indices: torch.Tensor,
                         weights: torch.Tensor, alpha: float, slots: int, saved: Optional[torch.Tensor] = None):
    """Gradients of slot_update: (grad_token_keys, grad_token_values, grad_old_slot_keys,
    grad_old_slot_values, grad_weights), the reference's slot_update_backward
    (torch_binding.cpp:19-21). ``saved`` is the forward's block; without it the per-slot means
    and weight sums are recomputed from the tokens, indices and weights."""
    lib = _lib.load_library()
    dt = token_keys.dtype
    tk = _rows(token_keys, dt)
    tv = _rows(token_values, dt)
    B, H, N, D = tk.shape
    M = int(slots)
    dev = tk.device
    gnk = _rows(grad_new_keys if grad_new_keys is not None else torch.zeros(B, H, M, D, device=dev, dtype=dt), dt)
    gnv = _rows(grad_new_values if grad_new_values is not None else torch.zeros(B, H, M, D, device=dev, dtype=dt), dt)
    idx = indices.to(device=dev, dtype=torch.int64).contiguous()
    w = weights.to(device=dev, dtype=torch.float32).contiguous()
    if saved is None:  # the means and weight sums do not depend on the old slot tables
        _, _, saved, _ = _update_forward(tk, tv, gnk, gnv, idx, w, alpha)
    shape = _shape(B, H, N, M, D, _DT[dt])
    _, ws_bytes = _sizes(shape)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    gtk = torch.empty(B, H, N, D, device=dev, dtype=dt)
    gtv = torch.empty(B, H, N, D, device=dev, dtype=dt)
    gsk = torch.empty(B, H, M, D, device=dev, dtype=dt)
    gsv = torch.empty(B, H, M, D, device=dev, dtype=dt)
    gw = torch.empty(B, H, N, 7, device=dev, dtype=torch.float32)
    a = _lib.SlotUpdateBwdArgs(
        shape=shape, alpha=float(alpha), token_keys=_ptr(tk), tk_stride=_s3(tk), token_values=_ptr(tv),
        tv_stride=_s3(tv), indices=_ptr(idx), weights=_ptr(w), saved=_ptr(saved), saved_bytes=saved.numel(),
        grad_new_keys=_ptr(gnk), gnk_stride=_s3(gnk), grad_new_values=_ptr(gnv), gnv_stride=_s3(gnv),
        grad_token_keys=_ptr(gtk), gtk_stride=_s3(gtk), grad_token_values=_ptr(gtv), gtv_stride=_s3(gtv),
        grad_slot_keys=_ptr(gsk), gsk_stride=_s3(gsk), grad_slot_values=_ptr(gsv), gsv_stride=_s3(gsv),
        grad_weights=_ptr(gw), workspace=_ptr(ws), workspace_bytes=ws_bytes)
    _lib.check(lib.murm_slot_update_bwd(ctypes.byref(a), _stream()))
    return gtk, gtv, gsk, gsv, gw


class _SlotUpdate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, token_keys, token_values, slot_keys, slot_values, indices, weights, alpha):
        nk, nv, saved, (tk, tv, idx, w) = _update_forward(token_keys, token_values, slot_keys, slot_values,
                                                           indices, weights, alpha)
        ctx.save_for_backward(tk, tv, idx, w, saved)
        ctx.alpha = float(alpha)
        ctx.M = slot_keys.shape[2]
        ctx.in_dtypes = (token_keys.dtype, token_values.dtype, slot_keys.dtype, slot_values.dtype)
        return nk, nv

    @staticmethod
    def backward(ctx, grad_nk, grad_nv):
        tk, tv, idx, w, saved = ctx.saved_tensors
        gtk, gtv, gsk, gsv, gw = slot_update_backward(grad_nk, grad_nv, tk, tv, idx, w, ctx.alpha, ctx.M, saved)
        a_t, b_t, c_t, d_t = ctx.in_dtypes
        return gtk.to(a_t), gtv.to(b_t), gsk.to(c_t), gsv.to(d_t), None, gw, None


class _SlotSums(torch.autograd.Function):
    @staticmethod
    def forward(ctx, token_keys, token_values, indices, weights, slots):
        ctx.M = int(slots)
        lib = _lib.load_library()
        code = _dtype_code(token_keys, "token_keys")
        dt = token_keys.dtype
        tk = _rows(token_keys, dt)
        tv = _rows(token_values, dt)
        B, H, N, D = tk.shape
        M = ctx.M
        shape = _shape(B, H, N, M, D, code)
        _, ws_bytes = _sizes(shape)
        dev = tk.device
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
        idx = indices.to(device=dev, dtype=torch.int64).contiguous()
        w = weights.to(device=dev, dtype=torch.float32).contiguous()
        ks = torch.empty(B, H, M, D, device=dev, dtype=torch.float32)
        vs = torch.empty(B, H, M, D, device=dev, dtype=torch.float32)
        ws_ = torch.empty(B, H, M, device=dev, dtype=torch.float32)
        a = _lib.SlotSumsArgs(shape=shape, token_keys=_ptr(tk), tk_stride=_s3(tk), token_values=_ptr(tv),
                              tv_stride=_s3(tv), indices=_ptr(idx), weights=_ptr(w), key_sums=_ptr(ks),
                              value_sums=_ptr(vs), weight_sums=_ptr(ws_), workspace=_ptr(ws),
                              workspace_bytes=ws_bytes)
        _lib.check(lib.murm_slot_sums_fwd(ctypes.byref(a), _stream()))
        ctx.save_for_backward(tk, tv, idx, w)
        ctx.in_dtypes = (token_keys.dtype, token_values.dtype)
        return ks, vs, ws_

    @staticmethod
    def backward(ctx, gks, gvs, gw_):
        lib = _lib.load_library()
        tk, tv, idx, w = ctx.saved_tensors
        B, H, N, D = tk.shape
        M = ctx.M
        dev = tk.device
        z = lambda *s: torch.zeros(*s, device=dev, dtype=torch.float32)
        gks = gks.float().contiguous() if gks is not None else z(B, H, M, D)
        gvs = gvs.float().contiguous() if gvs is not None else z(B, H, M, D)
        gw_ = gw_.float().contiguous() if gw_ is not None else z(B, H, M)
        gtk = torch.empty(B, H, N, D, device=dev, dtype=tk.dtype)
        gtv = torch.empty(B, H, N, D, device=dev, dtype=tk.dtype)
        gw = torch.empty(B, H, N, 7, device=dev, dtype=torch.float32)
        a = _lib.SlotSumsBwdArgs(shape=_shape(B, H, N, M, D, _DT[tk.dtype]), token_keys=_ptr(tk), tk_stride=_s3(tk),
                                 token_values=_ptr(tv), tv_stride=_s3(tv), indices=_ptr(idx), weights=_ptr(w),
                                 grad_key_sums=_ptr(gks), grad_value_sums=_ptr(gvs), grad_weight_sums=_ptr(gw_),
                                 grad_token_keys=_ptr(gtk), gtk_stride=_s3(gtk), grad_token_values=_ptr(gtv),
                                 gtv_stride=_s3(gtv), grad_weights=_ptr(gw))
        _lib.check(lib.murm_slot_sums_bwd(ctypes.byref(a), _stream()))
        a_t, b_t = ctx.in_dtypes
        return gtk.to(a_t), gtv.to(b_t), None, gw, None


def slot_diffusion_backward(grad_new_keys: torch.Tensor, grad_new_values: torch.Tensor,
                            gamma: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """The transposed stencil applied to the output gradients: the reference's
    slot_diffusion_backward (torch_binding.cpp:26-28)."""
    return _SlotDiffusion._run(_lib.load_library().murm_slot_diffusion_bwd, grad_new_keys, grad_new_values, gamma)


class _SlotDiffusion(torch.autograd.Function):
    @staticmethod
    def _run(fn, sk, sv, gamma):
        code = _dtype_code(sk, "slot_keys")
        dt = sk.dtype
        sk = _rows(sk, dt)
        sv = _rows(sv, dt)
        B, H, M, D = sk.shape
        ok = torch.empty(B, H, M, D, device=sk.device, dtype=dt)
        ov = torch.empty(B, H, M, D, device=sk.device, dtype=dt)
        a = _lib.SlotDiffusionArgs(shape=_shape(B, H, 1, M, D, code), gamma=float(gamma), in_keys=_ptr(sk),
                                   ik_stride=_s3(sk), in_values=_ptr(sv), iv_stride=_s3(sv), out_keys=_ptr(ok),
                                   ok_stride=_s3(ok), out_values=_ptr(ov), ov_stride=_s3(ov))
        _lib.check(fn(ctypes.byref(a), _stream()))
        return ok, ov

    @staticmethod
    def forward(ctx, slot_keys, slot_values, gamma):
        ctx.gamma = gamma
        return _SlotDiffusion._run(_lib.load_library().murm_slot_diffusion_fwd, slot_keys, slot_values, gamma)

    @staticmethod
    def backward(ctx, gk, gv):
        ref = gk if gk is not None else gv
        gk = gk if gk is not None else torch.zeros_like(ref)
        gv = gv if gv is not None else torch.zeros_like(ref)
        dk, dv = _SlotDiffusion._run(_lib.load_library().murm_slot_diffusion_bwd, gk, gv, ctx.gamma)
        return dk, dv, None


# ---------------------------------------------------------------------------
# The reference's public functions (ops.py)
# ---------------------------------------------------------------------------

def slot_select_attend(query: torch.Tensor, slot_keys: torch.Tensor, slot_values: torch.Tensor,
                       mask: Optional[torch.Tensor] = None, causal: bool = False,
                       position_bias: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                       effective_M: int = 0) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Select the 7 best slots per token and attend over them (ops.py:246-279)."""
    M = slot_keys.shape[2]
    em = effective_M if effective_M and effective_M > 0 else M
    return _SelectAttend.apply(query, slot_keys, slot_values, mask, causal, position_bias, scale, min(em, M), None)


def slot_select(query: torch.Tensor, slot_keys: torch.Tensor, mask: Optional[torch.Tensor] = None,
                causal: bool = False, position_bias: Optional[torch.Tensor] = None,
                effective_M: Optional[int] = None) -> torch.Tensor:
    """The top-7 slot indices per token (ops.py:219-236); int64 [B, H, N, 7]."""
    with torch.no_grad():
        _, _, idx = _SelectAttend.apply(query, slot_keys, slot_keys, mask, causal, position_bias, None,
                                        int(effective_M or 0), None)
    return idx


def slot_attend(query: torch.Tensor, slot_keys: torch.Tensor, slot_values: torch.Tensor, indices: torch.Tensor,
                scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Attend over given slot indices (ops.py:237-243; reference.py:42-68)."""
    out, w, _ = _SelectAttend.apply(query, slot_keys, slot_values, None, False, None, scale, 0, indices)
    return out, w


def slot_update(token_keys: torch.Tensor, token_values: torch.Tensor, slot_keys: torch.Tensor,
                slot_values: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor,
                alpha: float = 0.9) -> Tuple[torch.Tensor, torch.Tensor]:
    """EMA of every slot towards the weighted mean of the tokens that chose it (ops.py:282-308).
    Returns new tensors (the reference mutates clones of its inputs)."""
    return _SlotUpdate.apply(token_keys, token_values, slot_keys, slot_values, indices, weights, alpha)


def slot_sums(token_keys: torch.Tensor, token_values: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor,
              slots: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The first half of slot_update (reference.py:87-103): fp32 per-slot sums of the
    weighted token keys, token values and weights, ([B,H,M,d], [B,H,M,d], [B,H,M]).
    Differentiable. Sums over token shards add up (sequence parallelism)."""
    return _SlotSums.apply(token_keys, token_values, indices, weights, slots)


def slot_diffusion(slot_keys: torch.Tensor, slot_values: torch.Tensor,
                   gamma: float = 0.1) -> Tuple[torch.Tensor, torch.Tensor]:
    """One Jacobi step of the 3-point Laplacian along the slots (ops.py:311-327)."""
    return _SlotDiffusion.apply(slot_keys, slot_values, gamma)


def slot_murmurate(x: torch.Tensor, q_proj: torch.Tensor, k_proj: torch.Tensor, v_proj: torch.Tensor,
                   slot_k_emb: torch.Tensor, slot_v_emb: torch.Tensor, num_heads: int = 8, rounds: int = 3,
                   alpha: float = 0.9, gamma: float = 0.15, causal: bool = False,
                   mask: Optional[torch.Tensor] = None,
                   position_bias_fn: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                   use_dynamic_m: bool = True, slot_ratio: int = 8,
                   use_fused_update_diffuse: bool = True, return_slots: bool = False):
    """The reference's full round loop (ops.py:330-422): x, q/k/v projections [B, N, D],
    per-head slot embeddings [H, M, D/H] -> x + the rounds' attend outputs, [B, N, D].
    ``use_fused_update_diffuse`` is accepted for signature compatibility (update and
    diffusion are separate kernels here with identical results). With ``return_slots``
    the final slot tables [B, H, M, D/H] are returned too, ``(out, slot_k, slot_v)``: the
    prefill of a streaming decode (murmurative_attention_b200.decode)."""
    B, N, D = x.shape
    H = num_heads
    if D % H != 0:
        raise ValueError(f"Embedding dimension D ({D}) must be divisible by num_heads ({H})")
    Dh = D // H
    M = slot_k_emb.shape[1]
    effective_M = M
    if use_dynamic_m:                                   # ops.py:353-356
        effective_M = min(M, max(32, (N + slot_ratio - 1) // slot_ratio))
    x_h = x.view(B, N, H, Dh).permute(0, 2, 1, 3)
    q_h = q_proj.view(B, N, H, Dh).permute(0, 2, 1, 3)
    k_h = k_proj.view(B, N, H, Dh).permute(0, 2, 1, 3)
    v_h = v_proj.view(B, N, H, Dh).permute(0, 2, 1, 3)
    slot_k = slot_k_emb.unsqueeze(0).expand(B, H, M, Dh)
    slot_v = slot_v_emb.unsqueeze(0).expand(B, H, M, Dh)
    for _ in range(rounds):
        pos_bias = position_bias_fn(x_h) if position_bias_fn is not None else None
        attn_out, attn_w, indices = _SelectAttend.apply(q_h, slot_k, slot_v, mask, causal, pos_bias, None,
                                                        effective_M, None)
        x_h = x_h + attn_out
        slot_k, slot_v = _SlotUpdate.apply(k_h, v_h, slot_k, slot_v, indices, attn_w, alpha)
        slot_k, slot_v = _SlotDiffusion.apply(slot_k, slot_v, gamma)
    out = x_h.permute(0, 2, 1, 3).contiguous().view(B, N, D)
    return (out, slot_k, slot_v) if return_slots else out
