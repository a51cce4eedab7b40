"""C ABI checks that need no GPU: the library loads, exports every symbol
include/murm.h declares, its structs match the ctypes mirror, and argument
validation reports the documented status codes."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

from murmurative_attention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "murm.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MURM_API\s+[\w\s\*]+?\b(murm_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    declared = header_functions()
    assert declared, "no MURM_API declarations found"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in murm.h but not exported"
    assert sorted(_lib.EXPORTS) == declared


def test_abi_version():
    assert _lib.load_library().murm_abi_version() == 1


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "murm.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu %zu\\n\", sizeof(murm_shape), sizeof(murm_fwd_args),"
        " sizeof(murm_bwd_args), offsetof(murm_shape, alpha), offsetof(murm_fwd_args, saved),"
        " offsetof(murm_bwd_args, workspace)); return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    want = [ctypes.sizeof(_lib.Shape), ctypes.sizeof(_lib.FwdArgs), ctypes.sizeof(_lib.BwdArgs),
            _lib.Shape.alpha.offset, _lib.FwdArgs.saved.offset, _lib.BwdArgs.workspace.offset]
    assert [int(x) for x in got] == want


def _sizes(**kw):
    lib = _lib.load_library()
    base = dict(batch=1, heads=16, tokens=8192, slots=256, head_dim=64, rounds=3, top_k=7, causal=0,
                alpha=0.9, gamma=0.15, scale=0.0, dtype=_lib.MURM_F16)
    base.update(kw)
    s = _lib.Shape(**base)
    a, b, c = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    st = lib.murm_slot_murmurate_sizes(ctypes.byref(s), ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
    return st, a.value, b.value, c.value


def test_sizes_scale_with_problem():
    st, saved, fws, bws = _sizes()
    assert st == 0 and saved > 0 and fws > 0 and bws > 0
    st2, saved2, _, _ = _sizes(rounds=6)
    assert st2 == 0 and saved2 > saved


@pytest.mark.parametrize("kw,status", [
    (dict(top_k=5), 2),          # MURM_ERR_UNSUPPORTED: reference hard-codes k=7
    (dict(slots=6), 1),          # fewer slots than picks (torch.topk raises too)
    (dict(slots=300), 2),        # beyond one-byte slot indices
    (dict(head_dim=48), 2),
    (dict(tokens=0), 1),
    (dict(rounds=-1), 1),
    (dict(dtype=7), 3),          # MURM_ERR_DTYPE
])
def test_sizes_rejects_bad_shapes(kw, status):
    st, *_ = _sizes(**kw)
    assert st == status
    msg = _lib.load_library().murm_last_error_message().decode()
    assert msg


def test_null_args_rejected_without_gpu():
    lib = _lib.load_library()
    assert lib.murm_slot_murmurate_fwd(None, None) == 1
    assert lib.murm_slot_murmurate_bwd(None, None) == 1


def test_status_strings():
    lib = _lib.load_library()
    for code in range(7):
        assert lib.murm_status_string(code)


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_phase_struct_layout_matches_header(tmp_path):
    structs = [("murm_phase_shape", _lib.PhaseShape), ("murm_select_attend_args", _lib.SelectAttendArgs),
               ("murm_select_attend_bwd_args", _lib.SelectAttendBwdArgs),
               ("murm_slot_update_args", _lib.SlotUpdateArgs), ("murm_slot_update_bwd_args", _lib.SlotUpdateBwdArgs),
               ("murm_slot_diffusion_args", _lib.SlotDiffusionArgs), ("murm_decode_args", _lib.DecodeArgs),
               ("murm_slot_sums_args", _lib.SlotSumsArgs), ("murm_slot_sums_bwd_args", _lib.SlotSumsBwdArgs)]
    fields = [("murm_select_attend_args", "indices_in", _lib.SelectAttendArgs),
              ("murm_select_attend_args", "weights", _lib.SelectAttendArgs),
              ("murm_select_attend_bwd_args", "workspace_bytes", _lib.SelectAttendBwdArgs),
              ("murm_slot_update_args", "saved", _lib.SlotUpdateArgs),
              ("murm_slot_update_bwd_args", "grad_weights", _lib.SlotUpdateBwdArgs),
              ("murm_slot_diffusion_args", "out_values", _lib.SlotDiffusionArgs),
              ("murm_decode_args", "positions", _lib.DecodeArgs), ("murm_decode_args", "weights", _lib.DecodeArgs)]
    body = "".join(f'printf("%zu ", sizeof({c}));' for c, _ in structs)
    body += "".join(f'printf("%zu ", offsetof({c}, {f}));' for c, f, _ in fields)
    src = tmp_path / "phase.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "murm.h"\nint main(void){' + body + "return 0;}\n")
    exe = tmp_path / "phase"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    want = [ctypes.sizeof(s) for _, s in structs] + [getattr(s, f).offset for _, f, s in fields]
    assert got == want


def _phase_sizes(**kw):
    base = dict(batch=2, heads=4, tokens=128, slots=256, head_dim=64, dtype=_lib.MURM_F16)
    base.update(kw)
    s = _lib.PhaseShape(**base)
    a, b = ctypes.c_size_t(), ctypes.c_size_t()
    st = _lib.load_library().murm_phase_sizes(ctypes.byref(s), ctypes.byref(a), ctypes.byref(b))
    return st, a.value, b.value


def test_phase_sizes_and_validation():
    st, saved, ws = _phase_sizes()
    assert st == 0 and saved > 0 and ws > 0
    assert _phase_sizes(tokens=256)[2] > ws
    assert _phase_sizes(head_dim=128, slots=384)[0] == 0      # general path: d up to 128, M beyond 256
    for kw, status in [(dict(slots=6), 1), (dict(slots=2048), 2), (dict(head_dim=12), 2),
                       (dict(head_dim=256), 2), (dict(dtype=9), 3), (dict(batch=0), 1)]:
        assert _phase_sizes(**kw)[0] == status, kw


def test_phase_null_args_rejected_without_gpu():
    lib = _lib.load_library()
    for name in ("murm_select_attend_fwd", "murm_select_attend_bwd", "murm_slot_update_fwd", "murm_slot_update_bwd",
                 "murm_slot_diffusion_fwd", "murm_slot_diffusion_bwd", "murm_decode_step",
                 "murm_slot_sums_fwd", "murm_slot_sums_bwd"):
        assert getattr(lib, name)(None, None) == 1, name


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_host_step_struct_layout_matches_header(tmp_path):
    src = tmp_path / "host.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "murm.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu\\n\", sizeof(murm_host_step_args),"
        " offsetof(murm_host_step_args, grad_out), offsetof(murm_host_step_args, groups),"
        " offsetof(murm_host_step_args, workspace_bytes)); return 0;}\n")
    exe = tmp_path / "host"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    H = _lib.HostStepArgs
    assert got == [ctypes.sizeof(H), H.grad_out.offset, H.groups.offset, H.workspace_bytes.offset]


def test_host_step_sizes_and_validation():
    lib = _lib.load_library()
    shape = _lib.Shape(1, 16, 8192, 256, 64, 3, 7, 0, 0.9, 0.15, 0.0, _lib.MURM_F16)
    n1, n2 = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.murm_host_step_sizes(ctypes.byref(shape), 1, ctypes.byref(n1)) == 0
    assert lib.murm_host_step_sizes(ctypes.byref(shape), 4, ctypes.byref(n2)) == 0
    # full-size device copies of every input and output, plus one group's scratch
    io = 16 * 8192 * 64 * 2 * 4 + 16 * 256 * 64 * 2 * 4 + 16 * 8192 * 7 * (8 + 4)
    assert n1.value > io and io < n2.value < n1.value
    bad = _lib.Shape(1, 16, 8192, 256, 64, 3, 5, 0, 0.9, 0.15, 0.0, _lib.MURM_F16)
    assert lib.murm_host_step_sizes(ctypes.byref(bad), 0, ctypes.byref(n1)) == 2
    assert lib.murm_slot_murmurate_host_step(None, None) == 1
    args = _lib.HostStepArgs(shape)  # no buffers
    assert lib.murm_slot_murmurate_host_step(ctypes.byref(args), None) == 1
