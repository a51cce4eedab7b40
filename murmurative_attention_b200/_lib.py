"""ctypes binding of ``libmurm_b200.so`` (the C ABI in include/murm.h).

Replaces the reference's extension loader (src/murmurative/_cuda_kernels.py:
``ensure_compiled``): it loads the in-tree shared library once and raises
``RuntimeError`` when the library is missing or CUDA is unavailable. There is
no fallback path.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
# the in-tree build; MURM_B200_LIB names another build of the same library
LIB_PATH = os.environ.get("MURM_B200_LIB") or os.path.join(HERE, "libmurm_b200.so")

MURM_F32, MURM_F16, MURM_BF16 = 0, 1, 2
TOP_K = 7


class Shape(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("tokens", ctypes.c_int32),
        ("slots", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("rounds", ctypes.c_int32),
        ("top_k", ctypes.c_int32), ("causal", ctypes.c_int32),
        ("alpha", ctypes.c_double), ("gamma", ctypes.c_double), ("scale", ctypes.c_double),
        ("dtype", ctypes.c_int32),
    ]


Strides = ctypes.c_int64 * 3


class KernelTime(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 48), ("launches", ctypes.c_int64), ("total_ms", ctypes.c_double)]


class FwdArgs(ctypes.Structure):
    _fields_ = [
        ("shape", Shape),
        ("q", ctypes.c_void_p), ("q_stride", Strides),
        ("slots_k", ctypes.c_void_p), ("sk_stride", Strides),
        ("slots_v", ctypes.c_void_p), ("sv_stride", Strides),
        ("out", ctypes.c_void_p), ("out_stride", Strides),
        ("indices", ctypes.c_void_p),
        ("weights", ctypes.c_void_p),
        ("saved", ctypes.c_void_p), ("saved_bytes", ctypes.c_size_t),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class BwdArgs(ctypes.Structure):
    _fields_ = [
        ("shape", Shape),
        ("q", ctypes.c_void_p), ("q_stride", Strides),
        ("grad_out", ctypes.c_void_p), ("go_stride", Strides),
        ("grad_weights", ctypes.c_void_p),
        ("saved", ctypes.c_void_p), ("saved_bytes", ctypes.c_size_t),
        ("grad_q", ctypes.c_void_p), ("gq_stride", Strides),
        ("grad_slots_k", ctypes.c_void_p), ("gsk_stride", Strides),
        ("grad_slots_v", ctypes.c_void_p), ("gsv_stride", Strides),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


Strides4 = ctypes.c_int64 * 4


class PhaseShape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("slots", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32)]


class SelectAttendArgs(ctypes.Structure):
    _fields_ = [
        ("shape", PhaseShape), ("causal", ctypes.c_int32), ("effective_m", ctypes.c_int32),
        ("scale", ctypes.c_double),
        ("q", ctypes.c_void_p), ("q_stride", Strides),
        ("slot_keys", ctypes.c_void_p), ("sk_stride", Strides),
        ("slot_values", ctypes.c_void_p), ("sv_stride", Strides),
        ("mask", ctypes.c_void_p), ("mask_stride", Strides4),
        ("position_bias", ctypes.c_void_p), ("bias_stride", Strides4),
        ("indices_in", ctypes.c_void_p),
        ("out", ctypes.c_void_p), ("out_stride", Strides),
        ("indices", ctypes.c_void_p), ("weights", ctypes.c_void_p),
    ]


class SelectAttendBwdArgs(ctypes.Structure):
    _fields_ = [
        ("shape", PhaseShape), ("scale", ctypes.c_double),
        ("q", ctypes.c_void_p), ("q_stride", Strides),
        ("slot_keys", ctypes.c_void_p), ("sk_stride", Strides),
        ("slot_values", ctypes.c_void_p), ("sv_stride", Strides),
        ("indices", ctypes.c_void_p), ("weights", ctypes.c_void_p),
        ("grad_out", ctypes.c_void_p), ("go_stride", Strides),
        ("grad_weights", ctypes.c_void_p),
        ("grad_q", ctypes.c_void_p), ("gq_stride", Strides),
        ("grad_slot_keys", ctypes.c_void_p), ("gsk_stride", Strides),
        ("grad_slot_values", ctypes.c_void_p), ("gsv_stride", Strides),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class SlotUpdateArgs(ctypes.Structure):
    _fields_ = [
        ("shape", PhaseShape), ("alpha", ctypes.c_double),
        ("token_keys", ctypes.c_void_p), ("tk_stride", Strides),
        ("token_values", ctypes.c_void_p), ("tv_stride", Strides),
        ("slot_keys", ctypes.c_void_p), ("sk_stride", Strides),
        ("slot_values", ctypes.c_void_p), ("sv_stride", Strides),
        ("indices", ctypes.c_void_p), ("weights", ctypes.c_void_p),
        ("new_slot_keys", ctypes.c_void_p), ("nsk_stride", Strides),
        ("new_slot_values", ctypes.c_void_p), ("nsv_stride", Strides),
        ("saved", ctypes.c_void_p), ("saved_bytes", ctypes.c_size_t),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class SlotUpdateBwdArgs(ctypes.Structure):
    _fields_ = [
        ("shape", PhaseShape), ("alpha", ctypes.c_double),
        ("token_keys", ctypes.c_void_p), ("tk_stride", Strides),
        ("token_values", ctypes.c_void_p), ("tv_stride", Strides),
        ("indices", ctypes.c_void_p), ("weights", ctypes.c_void_p),
        ("saved", ctypes.c_void_p), ("saved_bytes", ctypes.c_size_t),
        ("grad_new_keys", ctypes.c_void_p), ("gnk_stride", Strides),
        ("grad_new_values", ctypes.c_void_p), ("gnv_stride", Strides),
        ("grad_token_keys", ctypes.c_void_p), ("gtk_stride", Strides),
        ("grad_token_values", ctypes.c_void_p), ("gtv_stride", Strides),
        ("grad_slot_keys", ctypes.c_void_p), ("gsk_stride", Strides),
        ("grad_slot_values", ctypes.c_void_p), ("gsv_stride", Strides),
        ("grad_weights", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class SlotDiffusionArgs(ctypes.Structure):
    _fields_ = [
        ("shape", PhaseShape), ("gamma", ctypes.c_double),
        ("in_keys", ctypes.c_void_p), ("ik_stride", Strides),
        ("in_values", ctypes.c_void_p), ("iv_stride", Strides),
        ("out_keys", ctypes.c_void_p), ("ok_stride", Strides),
        ("out_values", ctypes.c_void_p), ("ov_stride", Strides),
    ]


class SlotSumsArgs(ctypes.Structure):
    _fields_ = [
        ("shape", PhaseShape),
        ("token_keys", ctypes.c_void_p), ("tk_stride", Strides),
        ("token_values", ctypes.c_void_p), ("tv_stride", Strides),
        ("indices", ctypes.c_void_p), ("weights", ctypes.c_void_p),
        ("key_sums", ctypes.c_void_p), ("value_sums", ctypes.c_void_p), ("weight_sums", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class SlotSumsBwdArgs(ctypes.Structure):
    _fields_ = [
        ("shape", PhaseShape),
        ("token_keys", ctypes.c_void_p), ("tk_stride", Strides),
        ("token_values", ctypes.c_void_p), ("tv_stride", Strides),
        ("indices", ctypes.c_void_p), ("weights", ctypes.c_void_p),
        ("grad_key_sums", ctypes.c_void_p), ("grad_value_sums", ctypes.c_void_p),
        ("grad_weight_sums", ctypes.c_void_p),
        ("grad_token_keys", ctypes.c_void_p), ("gtk_stride", Strides),
        ("grad_token_values", ctypes.c_void_p), ("gtv_stride", Strides),
        ("grad_weights", ctypes.c_void_p),
    ]


Strides2 = ctypes.c_int64 * 2


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("slots", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32), ("causal", ctypes.c_int32),
        ("positions", ctypes.c_void_p),
        ("alpha", ctypes.c_double), ("gamma", ctypes.c_double), ("scale", ctypes.c_double),
        ("q", ctypes.c_void_p), ("q_stride", Strides2),
        ("k", ctypes.c_void_p), ("k_stride", Strides2),
        ("v", ctypes.c_void_p), ("v_stride", Strides2),
        ("x", ctypes.c_void_p), ("x_stride", Strides2),
        ("out", ctypes.c_void_p), ("out_stride", Strides2),
        ("slot_keys", ctypes.c_void_p), ("sk_stride", Strides),
        ("slot_values", ctypes.c_void_p), ("sv_stride", Strides),
        ("indices", ctypes.c_void_p), ("weights", ctypes.c_void_p),
    ]


class HostStepArgs(ctypes.Structure):
    _fields_ = [
        ("shape", Shape),
        ("q", ctypes.c_void_p), ("slots_k", ctypes.c_void_p), ("slots_v", ctypes.c_void_p),
        ("grad_out", ctypes.c_void_p), ("out", ctypes.c_void_p), ("indices", ctypes.c_void_p),
        ("weights", ctypes.c_void_p), ("grad_q", ctypes.c_void_p), ("grad_slots_k", ctypes.c_void_p),
        ("grad_slots_v", ctypes.c_void_p), ("groups", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


# Every symbol include/murm.h declares; tests check the library exports them all.
EXPORTS = (
    "murm_slot_murmurate_sizes",
    "murm_slot_murmurate_fwd",
    "murm_slot_murmurate_bwd",
    "murm_slot_murmurate_fwd_noscratch",
    "murm_slot_murmurate_fwd_f32_slots",
    "murm_status_string",
    "murm_last_error_message",
    "murm_abi_version",
    "murm_device_status",
    "murm_wait_probe",
    "murm_kernel_launches",
    "murm_profile_begin",
    "murm_profile_end",
    "murm_phase_sizes",
    "murm_select_attend_fwd",
    "murm_select_attend_bwd",
    "murm_slot_update_fwd",
    "murm_slot_update_bwd",
    "murm_slot_diffusion_fwd",
    "murm_slot_diffusion_bwd",
    "murm_decode_step",
    "murm_slot_sums_fwd",
    "murm_slot_sums_bwd",
    "murm_host_step_sizes",
    "murm_slot_murmurate_host_step",
)

STATUS_NAMES = {
    0: "MURM_OK", 1: "MURM_ERR_INVALID_ARGUMENT", 2: "MURM_ERR_UNSUPPORTED", 3: "MURM_ERR_DTYPE",
    4: "MURM_ERR_WORKSPACE", 5: "MURM_ERR_CUDA", 6: "MURM_ERR_DEVICE",
}

_lock = threading.Lock()
_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the shared library (no CUDA device needed) and declare prototypes."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"murmurative_attention_b200: CUDA library not built ({path} missing). "
                "Build it with:  python -m murmurative_attention_b200.build")
        lib = ctypes.CDLL(path)
        lib.murm_slot_murmurate_sizes.argtypes = [ctypes.POINTER(Shape), ctypes.POINTER(ctypes.c_size_t),
                                                  ctypes.POINTER(ctypes.c_size_t),
                                                  ctypes.POINTER(ctypes.c_size_t)]
        lib.murm_slot_murmurate_sizes.restype = ctypes.c_int
        lib.murm_slot_murmurate_fwd.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
        lib.murm_slot_murmurate_fwd.restype = ctypes.c_int
        lib.murm_slot_murmurate_bwd.argtypes = [ctypes.POINTER(BwdArgs), ctypes.c_void_p]
        lib.murm_slot_murmurate_bwd.restype = ctypes.c_int
        lib.murm_slot_murmurate_fwd_noscratch.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
        lib.murm_slot_murmurate_fwd_noscratch.restype = ctypes.c_int
        lib.murm_slot_murmurate_fwd_f32_slots.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
        lib.murm_slot_murmurate_fwd_f32_slots.restype = ctypes.c_int
        lib.murm_status_string.argtypes = [ctypes.c_int]
        lib.murm_status_string.restype = ctypes.c_char_p
        lib.murm_last_error_message.argtypes = []
        lib.murm_last_error_message.restype = ctypes.c_char_p
        lib.murm_abi_version.argtypes = []
        lib.murm_abi_version.restype = ctypes.c_int32
        lib.murm_device_status.argtypes = [ctypes.c_void_p]
        lib.murm_device_status.restype = ctypes.c_int
        lib.murm_wait_probe.argtypes = [ctypes.c_int32, ctypes.c_uint64, ctypes.c_void_p]
        lib.murm_wait_probe.restype = ctypes.c_int
        lib.murm_kernel_launches.argtypes = []
        lib.murm_kernel_launches.restype = ctypes.c_uint64
        lib.murm_profile_begin.argtypes = []
        lib.murm_profile_begin.restype = ctypes.c_int
        lib.murm_profile_end.argtypes = [ctypes.POINTER(KernelTime), ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
        lib.murm_profile_end.restype = ctypes.c_int
        lib.murm_phase_sizes.argtypes = [ctypes.POINTER(PhaseShape), ctypes.POINTER(ctypes.c_size_t),
                                         ctypes.POINTER(ctypes.c_size_t)]
        lib.murm_phase_sizes.restype = ctypes.c_int
        for name, st in (("murm_select_attend_fwd", SelectAttendArgs), ("murm_select_attend_bwd", SelectAttendBwdArgs),
                         ("murm_slot_update_fwd", SlotUpdateArgs), ("murm_slot_update_bwd", SlotUpdateBwdArgs),
                         ("murm_slot_diffusion_fwd", SlotDiffusionArgs),
                         ("murm_slot_diffusion_bwd", SlotDiffusionArgs), ("murm_decode_step", DecodeArgs),
                         ("murm_slot_sums_fwd", SlotSumsArgs), ("murm_slot_sums_bwd", SlotSumsBwdArgs)):
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.POINTER(st), ctypes.c_void_p]
            fn.restype = ctypes.c_int
        lib.murm_host_step_sizes.argtypes = [ctypes.POINTER(Shape), ctypes.c_int32, ctypes.POINTER(ctypes.c_size_t)]
        lib.murm_host_step_sizes.restype = ctypes.c_int
        lib.murm_slot_murmurate_host_step.argtypes = [ctypes.POINTER(HostStepArgs), ctypes.c_void_p]
        lib.murm_slot_murmurate_host_step.restype = ctypes.c_int
        if lib.murm_abi_version() != 1:
            raise RuntimeError("murmurative_attention_b200: libmurm_b200.so ABI version mismatch; rebuild it")
        _lib = lib
        return lib


class MurmError(RuntimeError):
    """A status other than MURM_OK from the C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def check(status: int) -> None:
    if status == 0:
        return
    msg = _lib.murm_last_error_message().decode() if _lib is not None else ""
    if status == 3:
        raise TypeError(msg)
    raise MurmError(status, msg)


def kernel_launches() -> int:
    """Kernels this library has launched in this process."""
    return int(load_library().murm_kernel_launches())


def profile_begin() -> None:
    check(load_library().murm_profile_begin())


def profile_end() -> dict:
    """{kernel name: (launches, total device ms)} since profile_begin()."""
    lib = load_library()
    cap = 64
    buf = (KernelTime * cap)()
    n = ctypes.c_int32()
    check(lib.murm_profile_end(buf, cap, ctypes.byref(n)))
    return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms)) for i in range(min(n.value, cap))}


def device_status(stream=None) -> None:
    """Synchronise ``stream`` and raise if a kernel reported a device-side error."""
    import torch
    st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    check(load_library().murm_device_status(ctypes.c_void_p(st)))
