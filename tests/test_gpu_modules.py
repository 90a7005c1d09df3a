"""GPU parity of the rac_torch module layer against the reference module.

tests/golden/rac_torch_block.npz holds the reference RACLlamaBlock
(rac_torch/rac_torch.py:1348-1383) run on CPU torch with seeded weights.
Our block loads the same state_dict and runs in FAST mode (the reference
module's default) on the GPU kernels.  Tolerance atol 1e-4, as the
reference's own RoPEAttention check (rac_torch/test_rac_dvt.py:865-894).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle as O
from rac_b200 import ext, tp
from rac_b200 import rac_torch as R

pytestmark = pytest.mark.gpu


def _block_from_golden(g, dev):
    d, H, ff, T, Bt, ms = [int(v) for v in g["cfg"]]
    blk = R.RACLlamaBlock(d, H, ff_dim=ff, max_seq_len=ms, activation="silu", bias=False).to(dev)
    sd = {k[2:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("w.")}
    missing, unexpected = blk.load_state_dict(sd, strict=False)
    assert not unexpected and all("cache" in m for m in missing), (missing, unexpected)
    return blk


@pytest.fixture
def fast_mode():
    R.rac_set_mode("fast")
    R.rac_set_precision(24)
    yield
    R.rac_set_mode("fast")


def test_llama_block_matches_reference_module(cuda, block_golden, fast_mode):
    blk = _block_from_golden(block_golden, cuda)
    x = torch.from_numpy(block_golden["x"]).to(cuda)
    with torch.no_grad():
        y = blk(x, is_causal=True).cpu().numpy()                  # fused-residual path
        y_nc = blk(x, is_causal=False).cpu().numpy()
    assert np.abs(y - block_golden["y"]).max() < 1e-4
    assert np.abs(y_nc - block_golden["y_noncausal"]).max() < 1e-4
    y_g = blk(x, is_causal=True).detach().cpu().numpy()          # autograd path
    assert np.abs(y_g - block_golden["y"]).max() < 1e-4


def test_rope_and_rmsnorm_match_reference(cuda, block_golden):
    blk = _block_from_golden(block_golden, cuda)
    q = torch.from_numpy(block_golden["rope_q"]).to(cuda)
    k = torch.from_numpy(block_golden["rope_k"]).to(cuda)
    rq, rk = blk.attn.rope(q, k)
    assert np.array_equal(rq.cpu().numpy(), block_golden["rope_q_out"])   # same rounding form
    assert np.array_equal(rk.cpu().numpy(), block_golden["rope_k_out"])
    n1 = blk.norm1(torch.from_numpy(block_golden["x"]).to(cuda)).detach().cpu().numpy()
    assert np.abs(n1 - block_golden["norm1"]).max() < 1e-5


def test_rope_positions(cuda):
    rope = R.RACRoPE(16, max_seq_len=32).to(cuda)
    q = torch.randn(1, 2, 5, 16, device=cuda)
    pos = torch.tensor([3, 7, 0, 31, 9], device=cuda)
    rq, _ = rope(q, q, positions=pos)
    c, s = rope.cos_cache[pos], rope.sin_cache[pos]
    x1, x2 = q[..., 0::2], q[..., 1::2]
    ref = torch.stack([x1 * c - x2 * s, x1 * s + x2 * c], -1).flatten(-2)
    assert torch.equal(rq, ref)


def test_linear_autograd_fast(cuda, fast_mode):
    torch.manual_seed(0)
    lin = R.RACLinear(48, 40).to(cuda)
    x = torch.randn(3, 7, 48, device=cuda, requires_grad=True)
    y = lin(x)
    y.square().sum().backward()
    xr = x.detach().clone().requires_grad_(True)
    w = lin.weight.detach().clone().requires_grad_(True)
    b = lin.bias.detach().clone().requires_grad_(True)
    yr = F.linear(xr, w, b)
    yr.square().sum().backward()
    assert torch.allclose(y, yr, atol=1e-5)
    assert torch.allclose(x.grad, xr.grad, atol=1e-4)
    assert torch.allclose(lin.weight.grad, w.grad, atol=1e-4)
    assert torch.allclose(lin.bias.grad, b.grad, atol=1e-4)


@pytest.mark.parametrize("act", ["relu", "gelu", "silu"])
def test_fused_linear_autograd(cuda, fast_mode, act):
    torch.manual_seed(1)
    lin = R.FusedRACLinear(32, 24, activation=act).to(cuda)
    x = torch.randn(5, 32, device=cuda, requires_grad=True)
    y = lin(x)
    y.sum().backward()
    xr = x.detach().clone().requires_grad_(True)
    w = lin.weight.detach().clone().requires_grad_(True)
    yr = {"relu": torch.relu, "gelu": F.gelu, "silu": F.silu}[act](F.linear(xr, w, lin.bias.detach()))
    yr.sum().backward()
    assert torch.allclose(y, yr, atol=1e-5)
    assert torch.allclose(x.grad, xr.grad, atol=1e-4) and torch.allclose(lin.weight.grad, w.grad, atol=1e-4)
    with torch.no_grad():
        assert torch.allclose(lin(x), yr, atol=1e-5)             # single fused kernel


def test_rac_matmul_cordic_mode_and_backward(cuda, orc):
    R.rac_set_mode("cordic")
    R.rac_set_precision(16)
    try:
        rng = np.random.default_rng(2)
        A = rng.uniform(-1, 1, (33, 45)).astype(np.float32)
        B = rng.uniform(-1, 1, (45, 29)).astype(np.float32)
        At = torch.from_numpy(A).to(cuda).requires_grad_(True)
        Bt = torch.from_numpy(B).to(cuda).requires_grad_(True)
        C = R.rac_matmul(At, Bt)
        assert np.array_equal(C.detach().cpu().numpy(), orc.gemm(A, B, "nn", 1, 16))
        G = torch.ones_like(C)
        C.backward(G)
        gA = orc.gemm(np.ones((33, 29), np.float32), np.ascontiguousarray(B), "nt", 1, 16)
        assert np.array_equal(At.grad.cpu().numpy(), gA)
    finally:
        R.rac_set_mode("fast")


def test_patch_model(cuda, fast_mode):
    m = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 8)).to(cuda)
    x = torch.randn(4, 16, device=cuda)
    ref = m(x)
    R.patch_model(m, False)                 # reference signature: (model, verbose, min_features=64)
    assert type(m[0]) is torch.nn.Linear and type(m[2]) is torch.nn.Linear
    R.patch_model(m, verbose=False, min_features=8)
    assert isinstance(m[0], R.RACLinear) and isinstance(m[2], R.RACLinear)
    assert torch.allclose(m(x), ref, atol=1e-5)
    R.unpatch_model(m, verbose=False)
    assert type(m[0]) is torch.nn.Linear


@pytest.mark.parametrize("mode", ["fast", "cordic"])
def test_tp_block_world1_equals_block(cuda, mode):
    R.rac_set_mode(mode)
    R.rac_set_precision(16)
    try:
        full = tp.make_block(128, 4, 344, 64, True, cuda, seed=5)
        x = torch.randn(2, 40, 128, device=cuda)
        with torch.no_grad():
            y = full(x, is_causal=True)
            y_tp = tp.TPLlamaBlock(full, 1, 0)(x)
        assert torch.equal(y, y_tp)
    finally:
        R.rac_set_mode("fast")


def test_tp_shard_transpose_follows_the_weight(cuda, fast_mode):
    """The FAST-mode W^T of a tensor-parallel shard is derived state: an in-place
    edit or a load_state_dict of the weight is seen by the next forward."""
    lin = tp._ShardLinear(torch.randn(24, 40, device=cuda))
    x = torch.randn(5, 40, device=cuda)
    want = lambda: ext.linear_forward(x, lin.weight, None, iters=24, mode=0)   # noqa: E731
    assert torch.equal(lin(x), want())
    with torch.no_grad():
        lin.weight.mul_(2)
    assert torch.equal(lin(x), want())
    lin.load_state_dict({"weight": torch.randn(24, 40, device=cuda)})
    assert torch.equal(lin(x), want())
    lin.weight.data = torch.randn(24, 40, device=cuda)
    assert torch.equal(lin(x), want())


def test_cpu_tensors_are_rejected():
    lin = R.RACLinear(4, 4)
    with pytest.raises(ValueError):
        lin(torch.randn(2, 4))


@pytest.mark.parametrize("mode,gated", [("fast", False), ("cordic", False), ("cordic", True)])
def test_llama_block_training_decreases_loss(cuda, mode, gated):
    """rac_torch/test_rac_dvt.py:897-923 (DVT-31): 20 Adam steps lower the loss by
    >= 5 %; every projection's forward and backward GEMM runs on the RAC kernels
    (NT forward, NN grad-input, TN grad-weight)."""
    R.rac_set_mode(mode)
    R.rac_set_precision(16)
    try:
        torch.manual_seed(0)
        block = R.RACLlamaBlock(d_model=32, n_heads=4, ff_dim=64, max_seq_len=16, gated=gated).to(cuda)
        opt = torch.optim.Adam(block.parameters(), lr=1e-3)
        x = torch.randn(2, 8, 32, device=cuda)
        target = torch.randn_like(x)
        losses = []
        for _ in range(20):
            opt.zero_grad()
            loss = (block(x, is_causal=True) - target).pow(2).mean()
            loss.backward()
            opt.step()
            losses.append(loss.item())
        assert losses[-1] < losses[0] * 0.95, losses
        with torch.no_grad():
            assert torch.isfinite(block(x)).all()
    finally:
        R.rac_set_mode("fast")
