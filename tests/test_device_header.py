"""include/rac_b200_device.cuh: the per-element device API.

CPU: the header compiles for sm_100a.  GPU: kernels built against it (nvcc at
test time, tests/c_client/dev_header_kernels.cu) return the bits of the
library's batch entry points -- rotate (literal RAC_K_INV), rotate_n,
project_n, sincos -- and a K-long chain of rac_dev_fma_cordic equals the
CORDIC GEMM's output (sequential k).
"""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "c_client", "dev_header_kernels.cu")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
         "-I", os.path.join(ROOT, "include")]


def _nvcc(args):
    if not os.path.exists(NVCC):
        pytest.skip("nvcc not available")
    r = subprocess.run([NVCC] + FLAGS + args, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_header_compiles_for_sm100a(tmp_path):
    _nvcc(["-c", SRC, "-o", str(tmp_path / "k.o")])


@pytest.mark.gpu
def test_device_api_matches_batch_entry_points(cuda, tmp_path):
    from rac_b200 import _lib, ext
    so = str(tmp_path / "libdevhdr.so")
    _nvcc(["-shared", "-Xcompiler", "-fPIC", SRC, "-o", so])
    L = ctypes.CDLL(so)
    vp, i = ctypes.c_void_p, ctypes.c_int
    L.run_elementwise.argtypes = [vp, vp, i, i, vp, vp, vp, vp, vp]
    L.run_dot.argtypes = [vp, vp, i, i, i, vp]
    rng = np.random.default_rng(11)
    n = 4099
    v = torch.from_numpy(rng.standard_normal((n, 2)).astype(np.float32)).to(cuda)
    th = torch.from_numpy(rng.uniform(-7, 7, n).astype(np.float32)).to(cuda)
    th[:6] = torch.tensor([0.0, -0.0, np.pi, -np.pi, float("nan"), 1.5707964])
    p = lambda t: t.data_ptr()                                   # noqa: E731
    for iters in (4, 8, 13, 16, 24):
        rot, rotn = torch.empty_like(v), torch.empty_like(v)
        proj, s, c = (torch.empty_like(th) for _ in range(3))
        assert L.run_elementwise(p(v), p(th), n, iters, p(rot), p(rotn), p(proj), p(s), p(c)) == 0
        same = lambda a, b: torch.equal(a.view(torch.int32), b.view(torch.int32))   # noqa: E731
        assert same(rot, ext.rotate_batch(v, th, None))
        assert same(rotn, ext.rotate_batch(v, th, iters))
        assert same(proj, ext.project_batch(v, th, iters))
        es, ec = ext.sincos(th)
        assert same(s, es) and same(c, ec)
    K = 96
    A = torch.from_numpy(rng.uniform(-1, 1, (n, K)).astype(np.float32)).to(cuda)
    b = torch.from_numpy(rng.uniform(-1, 1, K).astype(np.float32)).to(cuda)
    for iters in (5, 8, 16, 24):
        out = torch.empty(n, device=cuda)
        assert L.run_dot(p(A), p(b), n, K, iters, p(out)) == 0
        want = ext.gemm(A, b.view(K, 1), _lib.LAYOUT_NN, iters, 1)[:, 0]
        assert torch.equal(out, want), iters
