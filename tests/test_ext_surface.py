"""rac_b200.ext is a drop-in for the reference's compiled extension rac_cuda_ext.

The reference module rac_torch/rac_torch.py calls exactly these attributes of
its extension (rac_torch.py:100, :134-139, :183, :193, :229, :241, :423,
:465, :1056-1058, :1101-1103) with these keyword arguments
(rac_torch_bind.cpp:223-258, rac_torch.cu:1181-1214).  Runs on CPU: only the
surface is checked here; the GPU tests check the numbers.
"""
import inspect

from rac_b200 import ext

CALLS = {
    "matmul_forward": ["A", "B", "iters", "mode"],
    "matmul_backward": ["grad_C", "A", "B", "need_grad_A", "need_grad_B", "iters", "mode"],
    "linear_forward": ["input", "weight", "bias", "iters", "mode"],
    "linear_backward": ["grad_output", "input", "weight", "need_bias_grad", "iters", "mode"],
    "fused_linear_forward": ["input", "weight", "bias", "act"],
    "fused_linear_backward": ["grad_output", "input", "weight", "bias", "pre_act", "act", "has_bias"],
    "set_cordic_iters": ["iters"],
    "set_cordic_mode": ["mode"],
    "get_cordic_iters": [],
    "get_cordic_mode": [],
}


def test_every_called_attribute_exists_with_its_arguments():
    for name, args in CALLS.items():
        fn = getattr(ext, name)
        params = list(inspect.signature(fn).parameters)
        assert params[:len(args)] == args, (name, params)


def test_defaults_match_the_binding():
    sig = inspect.signature(ext.matmul_forward)
    assert sig.parameters["iters"].default == 0 and sig.parameters["mode"].default == -1
    sig = inspect.signature(ext.matmul_backward)
    assert sig.parameters["need_grad_A"].default is True and sig.parameters["need_grad_B"].default is True
    assert (ext.MODE_FAST, ext.MODE_CORDIC, ext.MODE_SHIFTADD) == (0, 1, 2)


def test_knob_semantics():
    ext.set_cordic_iters(0)
    assert ext.get_cordic_iters() == 24          # <= 0 resets (rac_torch_bind.cpp:205-212)
    ext.set_cordic_iters(99)
    assert ext.get_cordic_iters() == 24
    ext.set_cordic_iters(7)
    assert ext.get_cordic_iters() == 7
    ext.set_cordic_mode(5)
    assert ext.get_cordic_mode() == ext.MODE_FAST    # unknown -> FAST (:216-219)
    ext.set_cordic_mode(ext.MODE_CORDIC)
    assert ext.get_cordic_mode() == ext.MODE_CORDIC
    ext.set_cordic_mode(ext.MODE_FAST)
    ext.set_cordic_iters(0)
