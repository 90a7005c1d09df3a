"""The unmodified reference module (rac_torch/rac_torch.py) running on this
library: ``rac_b200.ext`` installed as ``rac_cuda_ext`` -- the import the
reference makes at rac_torch.py:42 -- and the reference's own classes driven
on CUDA tensors.

`oracle.build()` places a copy of the reference module under
oracle/_ref/py/ (git-ignored, built from the reference checkout); without it
the tests skip.  What is checked:

* the reference's import-time probes (rac_torch.py:62-151) find the extension
  working and accepting the per-call ``iters`` / ``mode`` kwargs;
* its knobs (rac_set_precision / rac_set_mode, :1038-1118) reach this
  library's process-wide knobs;
* its RACLinear, FusedRACLinear and rac_matmul, forward and backward, give
  the same bits as rac_b200.rac_torch in FAST, CORDIC-16 and SHIFTADD mode;
* its RACLlamaBlock forward (attention core in torch.matmul / torch.softmax,
  projections on this library) matches rac_b200's block within 1e-4.
"""
import importlib.util
import os
import sys

import pytest
import torch

import oracle as O
from rac_b200 import ext
from rac_b200 import rac_torch as R

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(os.path.join(O.REF_PY_DIR, "rac_torch_ref.py")),
                                 reason="reference module copy not built (oracle.build())")]


@pytest.fixture(scope="module")
def ref_mod(cuda):
    saved = sys.modules.get("rac_cuda_ext")
    sys.modules["rac_cuda_ext"] = ext
    spec = importlib.util.spec_from_file_location("rac_torch_ref",
                                                  os.path.join(O.REF_PY_DIR, "rac_torch_ref.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    yield mod
    if saved is None:
        sys.modules.pop("rac_cuda_ext", None)
    else:
        sys.modules["rac_cuda_ext"] = saved
    R.rac_set_mode("fast")
    R.rac_set_precision(24)


def _both(ref_mod, mode, iters):
    ref_mod.rac_set_mode(mode)
    ref_mod.rac_set_precision(iters)
    R.rac_set_mode(mode)
    R.rac_set_precision(iters)


def test_reference_probes_accept_this_library(ref_mod):
    assert ref_mod._rac_available()
    assert ref_mod._RAC_ACCEPTS_ITERS and ref_mod._RAC_ACCEPTS_MODE
    assert ref_mod._rac_has("fused_linear_forward")
    ref_mod.rac_set_mode("cordic")
    ref_mod.rac_set_precision(12)
    assert ext.get_cordic_mode() == ext.MODE_CORDIC and ext.get_cordic_iters() == 12


@pytest.mark.parametrize("mode,iters", [("fast", 24), ("cordic", 16), ("shiftadd", 8)])
def test_reference_linear_and_matmul_same_bits(ref_mod, cuda, mode, iters):
    _both(ref_mod, mode, iters)
    torch.manual_seed(1)
    theirs = ref_mod.RACLinear(96, 80).to(cuda)
    ours = R.RACLinear(96, 80).to(cuda)
    ours.load_state_dict(theirs.state_dict())
    x = torch.randn(4, 9, 96, device=cuda)
    xa = x.clone().requires_grad_(True)
    xb = x.clone().requires_grad_(True)
    ya, yb = theirs(xa), ours(xb)
    assert torch.equal(ya, yb)
    g = torch.randn_like(ya)
    ya.backward(g)
    yb.backward(g)
    assert torch.equal(xa.grad, xb.grad)
    assert torch.equal(theirs.weight.grad, ours.weight.grad)
    assert torch.equal(theirs.bias.grad, ours.bias.grad)
    A = torch.randn(33, 70, device=cuda)
    B = torch.randn(70, 41, device=cuda)
    assert torch.equal(ref_mod.rac_matmul(A, B), R.rac_matmul(A, B))


@pytest.mark.parametrize("mode,iters", [("fast", 24), ("cordic", 16)])
def test_reference_fused_linear_same_bits(ref_mod, cuda, mode, iters):
    _both(ref_mod, mode, iters)
    torch.manual_seed(2)
    theirs = ref_mod.FusedRACLinear(64, 48, activation="silu").to(cuda)
    ours = R.FusedRACLinear(64, 48, activation="silu").to(cuda)
    ours.load_state_dict(theirs.state_dict())
    x = torch.randn(5, 64, device=cuda)
    with torch.no_grad():
        assert torch.equal(theirs(x), ours(x))


@pytest.mark.parametrize("mode,iters", [("fast", 24), ("cordic", 16)])
def test_reference_llama_block_on_this_library(ref_mod, cuda, mode, iters):
    _both(ref_mod, mode, iters)
    torch.manual_seed(3)
    d, H, ff, T = 256, 4, 704, 64
    theirs = ref_mod.RACLlamaBlock(d, H, ff_dim=ff, max_seq_len=T).to(cuda)
    ours = R.RACLlamaBlock(d, H, ff_dim=ff, max_seq_len=T).to(cuda)
    missing, unexpected = ours.load_state_dict(theirs.state_dict(), strict=False)
    assert not unexpected and all("cache" in m for m in missing)
    x = torch.randn(2, T, d, device=cuda)
    with torch.no_grad():
        ya = theirs(x, is_causal=True)
        yb = ours(x, is_causal=True)
    scale = ya.pow(2).mean().sqrt().item()
    assert (ya - yb).abs().max().item() <= 1e-4 * scale
