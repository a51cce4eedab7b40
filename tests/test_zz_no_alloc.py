"""The forward entry point that allocates nothing (murm_slot_murmurate_fwd_noscratch).

Some callers cannot allocate device memory — a serving plugin handed only its
input and output buffers under a fixed memory budget, or a foreign-language
host without a binding to the CUDA allocator. For them the library keeps its forward scratch in one
built-in 64 MiB device array. These tests call that entry point through the C
ABI and check it against the regular entry point (caller-provided scratch) on
two calls in a row with different inputs, so contents the shared array keeps
from the previous call cannot leak into the next result. This file sorts last
so that a run stopping at its first failure has run every other test.
"""
import ctypes

import pytest
import torch

from murmurative_attention_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _inputs(seed, B=1, H=4, N=2048, D=64, M=256, dtype=torch.float16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g, device="cuda").to(dtype)
    sk = torch.randn(B, H, M, D, generator=g, device="cuda").to(dtype)
    sv = (torch.randn(B, H, M, D, generator=g, device="cuda") * 0.1).to(dtype)
    return q, sk, sv


def _args(q, sk, sv, rounds=3, causal=False, saved=None, ws=None):
    shape = ops._make_shape(q, sk.shape[2], rounds, 7, causal, 0.9, 0.15, None)
    B, H, N, _ = q.shape
    out = torch.full_like(q, float("nan"))
    idx = torch.full((B, H, N, 7), -1, dtype=torch.int64, device="cuda")
    w = torch.full((B, H, N, 7), float("nan"), dtype=torch.float32, device="cuda")
    S = ops._strides
    a = _lib.FwdArgs(shape, q.data_ptr(), S(q), sk.data_ptr(), S(sk), sv.data_ptr(), S(sv), out.data_ptr(), S(out),
                     idx.data_ptr(), w.data_ptr(), saved.data_ptr() if saved is not None else None,
                     saved.numel() if saved is not None else 0, ws.data_ptr() if ws is not None else None,
                     ws.numel() if ws is not None else 0)
    return a, shape, (out, idx, w)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _regular(q, sk, sv, causal):
    lib = _lib.load_library()
    shape = ops._make_shape(q, sk.shape[2], 3, 7, causal, 0.9, 0.15, None)
    saved_b, fws_b, _ = ops.slot_murmurate_sizes(shape)
    saved = torch.empty(saved_b, dtype=torch.uint8, device="cuda")
    ws = torch.empty(fws_b, dtype=torch.uint8, device="cuda")
    a, _, res = _args(q, sk, sv, causal=causal, saved=saved, ws=ws)
    _lib.check(lib.murm_slot_murmurate_fwd(ctypes.byref(a), _stream()))
    return res


@pytest.mark.parametrize("causal", [False, True])
def test_noscratch_forward_matches_regular_forward_twice(causal):
    lib = _lib.load_library()
    for call, seed in enumerate((11, 12)):
        q, sk, sv = _inputs(seed)
        ref_out, ref_idx, ref_w = _regular(q, sk, sv, causal)
        a, _, (out, idx, w) = _args(q, sk, sv, causal=causal)
        _lib.check(lib.murm_slot_murmurate_fwd_noscratch(ctypes.byref(a), _stream()))
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx), f"call {call}: indices differ"
        torch.testing.assert_close(out.float(), ref_out.float(), atol=2e-3, rtol=1e-2)
        torch.testing.assert_close(w, ref_w, atol=2e-3, rtol=1e-2)


def test_noscratch_rejects_problems_beyond_its_scratch():
    lib = _lib.load_library()
    q, sk, sv = _inputs(0, B=1, H=64, N=8192)
    a, shape, _ = _args(q, sk, sv)
    saved_b, fws_b, _ = ops.slot_murmurate_sizes(shape)
    assert saved_b + fws_b > (64 << 20)
    st = lib.murm_slot_murmurate_fwd_noscratch(ctypes.byref(a), _stream())
    assert st == 4  # MURM_ERR_WORKSPACE
    assert b"built-in scratch" in lib.murm_last_error_message()


def test_noscratch_refuses_caller_scratch():
    lib = _lib.load_library()
    q, sk, sv = _inputs(1, N=256)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    a, _, _ = _args(q, sk, sv, ws=ws)
    assert lib.murm_slot_murmurate_fwd_noscratch(ctypes.byref(a), _stream()) == 1
