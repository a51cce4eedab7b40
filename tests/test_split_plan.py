"""The forward's (b,h) x tile split plan (murm_common.cuh: TileSplit, plan_split, max_parts),
checked on the host by a small C++ program compiled against the same header (host code only: it
runs without a GPU)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    return None


def test_split_plan_invariants(tmp_path):
    nvcc = _nvcc()
    if not nvcc:
        pytest.skip("needs nvcc")
    exe = str(tmp_path / "split_plan_check")
    subprocess.run([nvcc, "-std=c++17", "-O1", "-x", "cu", "-I", os.path.join(HERE, "..", "include"),
                    os.path.join(HERE, "split_plan_check.cpp"), "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr
