"""RACLlamaBlock at the benchmark's configuration -- d_model 4096, 32 heads,
head_dim 128, ff_dim 11008, RMSNorm eps 1e-6, RoPE base 1e4, causal -- in
FAST and CORDIC-16 mode, with the SwiGLU FFN the tokens/s benchmark runs
(bench/bench_rac_transformer.c:441-453) and with the reference module's own
SiLU FFN (rac_torch/rac_torch.py:1348-1383, :631-655).

The checker is oracle/torch_block.py (the reference module's CPU path in
plain fp32 torch), on x [1, 256, 4096] with the benchmark's weight init.  In
CORDIC mode each projection's activation operand first goes through
oracle.cordic_operand: the CORDIC-mode MAC is fmaf(r(a), w, acc) exactly,
so the CPU checker then differs from the GPU only by summation order.

Bar: max |y - y_ref| <= 1e-4 * rms(y_ref), the 1e-4 the reference's own
module checks use (rac_torch/test_rac_dvt.py:757-796).  The single-GPU
tensor-parallel shard (the code the benchmark times) must equal the module's
output bit for bit (its FAST projections run NN on a cached W^T, the
module's NT on W: the same fma sequence per output).
"""
import numpy as np
import pytest
import torch

import oracle as O
from oracle import torch_block as TB
from rac_b200 import rac_torch as R
from rac_b200 import tp

pytestmark = pytest.mark.gpu

D, H, FF, T = 4096, 32, 11008, 256
TOL = 1e-4


@pytest.fixture
def restore_mode():
    yield
    R.rac_set_mode("fast")
    R.rac_set_precision(24)


def _operand(mode, iters):
    if mode != "cordic":
        return None
    return lambda t: torch.from_numpy(O.cordic_operand(t.contiguous().numpy(), iters))


@pytest.mark.parametrize("gated", [True, False])
@pytest.mark.parametrize("mode", ["fast", "cordic"])
def test_block_at_benchmark_config(cuda, restore_mode, gated, mode):
    iters = 16
    R.rac_set_mode(mode)
    R.rac_set_precision(iters)
    blk = tp.make_block(D, H, FF, T, gated, cuda, seed=11)
    g = torch.Generator().manual_seed(12)
    x = torch.randn((1, T, D), generator=g)
    xd = x.to(cuda)
    with torch.no_grad():
        y_mod = blk(xd, is_causal=True)
        shard = tp.TPLlamaBlock(blk, 1, 0)
        y_tp = shard(xd)
    assert torch.equal(y_tp, y_mod), "tensor-parallel shard differs from the module"
    p = TB.params_of(blk)
    del shard, blk
    torch.cuda.empty_cache()
    with torch.no_grad():
        cos, sin = TB.rope_cache(D // H, T)
        ref = TB.block_forward(p, x, H, cos=cos, sin=sin, operand=_operand(mode, iters)).numpy()
    y = y_mod.cpu().numpy()
    scale = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    err = float(np.abs(y - ref).max()) / scale
    print(f"block d={D} gated={gated} {mode}: max|diff|/rms = {err:.3e}")
    assert err <= TOL, err
    if mode == "cordic":
        # the CORDIC projections are not the FAST ones: the checker must see it
        with torch.no_grad():
            plain = TB.block_forward(p, x, H, cos=cos, sin=sin).numpy()
        assert np.abs(plain - ref).max() > 0
