"""The reference's own acceptance checks for this path, on the GPU library.

* DVT-11 (lib/c/test_rac_lib_dvt.c:354-382): rsqrt over [0.5, 64] within 1e-4
  of 1/sqrtf, rsqrt(0) == 0, sigmoid over [-5, 5] within 1e-5 of
  1/(1+expf(-x)), sincos on the full circle within 0.01 of libm -- through
  the scalar rac.h entry points.
* DVT-1 (rac_torch/test_rac_dvt.py:67-97): rac_matmul shape sweep against
  torch.matmul with tol = max(1e-2, K * 1e-5), in FAST and CORDIC-16 mode.
* E2E-18 (rac_torch/test_rac_e2e.py:697-723): RACLlamaBlock(64, 8, ff 128)
  trained 60 Adam steps (lr 1e-3) reaches loss < 0.85 x the first step's.
"""
import ctypes
import math

import pytest
import torch

from rac_b200 import _lib
from rac_b200 import rac_torch as R

pytestmark = pytest.mark.gpu


def test_dvt11_rsqrt_sigmoid_sincos(cuda):
    L = _lib.lib()
    for i in range(1, 129):
        x = i * 0.5
        assert abs(L.rac_rsqrt(ctypes.c_float(x)) - 1.0 / math.sqrt(x)) <= 1e-4
    assert L.rac_rsqrt(ctypes.c_float(0.0)) == 0.0
    for i in range(-20, 21):
        x = i * 0.25
        assert abs(L.rac_sigmoid(ctypes.c_float(x)) - 1.0 / (1.0 + math.exp(-x))) <= 1e-5
    s, c = ctypes.c_float(), ctypes.c_float()
    for deg in range(0, 360, 11):
        th = deg * 3.14159265358979 / 180.0
        L.rac_sincos(ctypes.c_float(th), ctypes.addressof(s), ctypes.addressof(c))
        assert abs(s.value - math.sin(th)) <= 0.01 and abs(c.value - math.cos(th)) <= 0.01
    _lib.check()


@pytest.mark.parametrize("mode", ["fast", "cordic"])
def test_dvt1_matmul_shape_sweep(cuda, mode):
    shapes = [(1, 1, 1), (1, 64, 1), (1, 1, 64), (16, 16, 16), (32, 64, 128), (128, 64, 32),
              (63, 65, 67), (127, 255, 131), (256, 256, 256), (512, 1024, 512), (1024, 1024, 1024),
              (1, 4096, 1), (4096, 1, 4096)]
    R.rac_set_mode(mode)
    R.rac_set_precision(16)
    try:
        g = torch.Generator(device=cuda).manual_seed(42)
        for M, K, N in shapes:
            A = torch.randn((M, K), device=cuda, generator=g)
            B = torch.randn((K, N), device=cuda, generator=g)
            err = (torch.matmul(A, B) - R.rac_matmul(A, B)).abs().max().item()
            assert err < max(1e-2, K * 1e-5), (M, K, N, err)
    finally:
        R.rac_set_mode("fast")
        R.rac_set_precision(24)


def test_e2e18_llama_block_training(cuda):
    R.rac_set_mode("fast")
    torch.manual_seed(0)
    block = R.RACLlamaBlock(d_model=64, n_heads=8, ff_dim=128, max_seq_len=32).to(cuda)
    opt = torch.optim.Adam(block.parameters(), lr=1e-3)
    x = torch.randn(4, 16, 64, device=cuda)
    target = torch.randn_like(x)
    losses = []
    for _ in range(60):
        opt.zero_grad()
        loss = (block(x, is_causal=True) - target).pow(2).mean()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0] * 0.85, (losses[0], losses[-1])
