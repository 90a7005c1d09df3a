"""A plain C program written against include/rac.h links librac_b200.so.

CPU: it compiles and links with gcc, and without a device every call reports
RAC_ERR_CUDA (exit 2) instead of computing on the CPU.  GPU: it runs and its
results match plain C loops (exit 0).
"""
import os
import subprocess

import pytest

from rac_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_client", "rac_client.c")


def _build(tmp_path):
    exe = str(tmp_path / "rac_client")
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["gcc", "-O2", "-std=c99", "-I", os.path.join(ROOT, "include"), SRC, "-o", exe,
                    "-L", libdir, "-lrac_b200", f"-Wl,-rpath,{libdir}", "-lm"],
                   check=True, capture_output=True, text=True)
    return exe


def test_c_client_builds_and_reports_missing_device(tmp_path):
    exe = _build(tmp_path)
    if _lib.lib().rac_b200_device_count() > 0:
        pytest.skip("a device is present (the GPU test runs the client)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 2, r.stdout + r.stderr


@pytest.mark.gpu
def test_c_client_runs_on_gpu(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
