"""The expert-parallel combine's epoch words are 32-bit and wrap; this builds
the header's epoch helpers on the host and walks them across the signed and
unsigned 32-bit limits (a wrapped epoch must neither accept a stale flag nor
reject the current one)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_epoch_wraps_safely(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    cuda_inc = "/usr/local/cuda/include"
    exe = str(tmp_path / "ep_epoch_check")
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "strataflow_b200", "csrc"), "-I", cuda_inc,
                    os.path.join(ROOT, "tests", "ep_epoch_check.cpp"), "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.startswith("ok")
