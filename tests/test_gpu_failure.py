"""Failure detection on the GPU without a fault: a bounded device wait that runs out.

Every mbarrier wait of the tensor-core kernels is bounded; on expiry a kernel sets the device
error word, skips its remaining work and returns, and murm_device_status turns the word into
MURM_ERR_DEVICE. murm_wait_probe runs that same bounded wait in a one-block kernel on a barrier
that nothing arrives on (a short limit), so the expiry path is exercised with no trap, no fault
and no hang; the context must stay usable afterwards.
"""
import ctypes

import pytest
import torch

from murmurative_attention_b200 import _lib, slot_murmurate

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_wait_that_completes_reports_nothing():
    lib = _lib.load_library()
    _lib.device_status()  # start from a clear error word
    _lib.check(lib.murm_wait_probe(1, 2_000_000, _stream()))
    _lib.device_status()


def test_expired_wait_is_reported_and_the_context_survives():
    lib = _lib.load_library()
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(1, 2, 300, 64, device="cuda", generator=g).half()
    sk = torch.randn(1, 2, 256, 64, device="cuda", generator=g).half()
    sv = torch.zeros_like(sk)
    before = slot_murmurate(q, sk, sv, rounds=3)
    _lib.device_status()
    _lib.check(lib.murm_wait_probe(0, 2_000_000, _stream()))  # nothing arrives: 2 ms, then give up
    with pytest.raises(_lib.MurmError) as err:
        _lib.device_status()
    assert err.value.status == 6  # MURM_ERR_DEVICE
    assert "0x10" in str(err.value)
    _lib.device_status()  # the word was read and cleared
    after = slot_murmurate(q, sk, sv, rounds=3)  # the context still runs the op
    _lib.device_status()
    for a, b in zip(before, after):
        assert torch.equal(a, b)


def test_probe_rejects_unbounded_limits():
    lib = _lib.load_library()
    assert lib.murm_wait_probe(0, 0, _stream()) == 1
    assert lib.murm_wait_probe(0, 11_000_000_000, _stream()) == 1
