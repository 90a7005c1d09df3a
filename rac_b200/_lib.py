"""ctypes binding of librac_b200.so (the C ABI in include/rac.h and rac_b200.h).

The library is loaded RTLD_LOCAL from the package directory.  A missing
library is an error, never a fallback: ``lib()`` raises ``RacError``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librac_b200.so")

RAC_OK = 0
STATUS_NAMES = {
    0: "RAC_OK", -1: "RAC_ERR_NULL_PTR", -2: "RAC_ERR_INVALID_DIM", -3: "RAC_ERR_ALLOC",
    -4: "RAC_ERR_CUDA", -5: "RAC_ERR_UNSUPPORTED", -6: "RAC_ERR_DEVICE",
}

LAYOUT_NN, LAYOUT_NT, LAYOUT_TN = 0, 1, 2
UNARY_EXP, UNARY_TANH, UNARY_RSQRT, UNARY_SIGMOID = 0, 1, 2, 3


class RacError(RuntimeError):
    """A librac_b200 call returned a non-zero status."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class Float2(C.Structure):
    _fields_ = [("x", C.c_float), ("y", C.c_float)]


_lock = threading.Lock()
_lib = None

_vp, _i, _ll, _f = C.c_void_p, C.c_int, C.c_longlong, C.c_float

# name -> (restype, argtypes)
_SIGS = {
    "rac_last_error": (_i, []),
    "rac_last_error_string": (C.c_char_p, []),
    "rac_clear_error": (None, []),
    "rac_set_cordic_iters": (None, [_i]),
    "rac_get_cordic_iters": (_i, []),
    "rac_set_cordic_mode": (None, [_i]),
    "rac_get_cordic_mode": (_i, []),
    "rac_b200_version": (C.c_char_p, []),
    "rac_b200_device_count": (_i, []),
    "rac_b200_cordic_gemm_directions": (None, [_vp]),
    "rac_create_context": (_vp, [_i]),
    "rac_destroy_context": (None, [_vp]),
    "rac_query_capability": (_i, [_vp, _i]),
    "rac_execute": (_i, [_vp, _i, _vp]),
    "rac_rotate": (Float2, [Float2, _f]),
    "rac_rotate_precision": (Float2, [Float2, _f, _i]),
    "rac_project_precision": (_f, [Float2, _f, _i]),
    "rac_exp": (_f, [_f]),
    "rac_tanh": (_f, [_f]),
    "rac_rsqrt": (_f, [_f]),
    "rac_sigmoid": (_f, [_f]),
    "rac_sincos": (None, [_f, _vp, _vp]),
    "rac_softmax": (None, [_vp, _vp, _i]),
    "rac_softmax_batch": (None, [_vp, _vp, _i, _i]),
    "rac_rotate_batch": (None, [_vp, _vp, _vp, _i]),
    "rac_rotate_batch_n": (None, [_vp, _vp, _vp, _i, _i]),
    "rac_project_batch_n": (None, [_vp, _vp, _vp, _i, _i]),
    "rac_exp_batch": (None, [_vp, _vp, _i]),
    "rac_tanh_batch": (None, [_vp, _vp, _i]),
    "rac_rsqrt_batch": (None, [_vp, _vp, _i]),
    "rac_sigmoid_batch": (None, [_vp, _vp, _i]),
    "rac_sincos_batch": (None, [_vp, _vp, _vp, _i]),
    "rac_matmul": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "rac_matmul_ex": (None, [_vp, _vp, _vp, _i, _i, _i, _i, _i]),
    "rac_rmsnorm": (None, [_vp, _vp, _vp, _f, _i, _i]),
    "rac_layernorm": (None, [_vp, _vp, _vp, _vp, _f, _i, _i]),
    "rac_rope_cache": (None, [_vp, _vp, _i, _i, _f]),
    "rac_rope_apply": (None, [_vp, _vp, _vp, _i, _i, _i, _i]),
    "rac_launch_nn_iters": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _i, _i, _vp]),
    "rac_launch_nt_iters": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _i, _i, _vp]),
    "rac_launch_tn_iters": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _i, _i, _vp]),
    "rac_launch_nn": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _vp]),
    "rac_launch_nt": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _vp]),
    "rac_launch_tn": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _vp]),
    "rac_gemm_async": (_i, [_vp, _ll, _vp, _ll, _vp, _ll, _vp, _ll, _vp, _i, _i, _i,
                            _i, _i, _i, _f, _f, _i, _i, _vp]),
    "rac_gemm_splitk_noalloc_async": (_i, [_vp, _ll, _vp, _ll, _vp, _ll, _vp, _ll, _vp, _i, _i,
                                           _i, _i, _i, _i, _f, _f, _i, _i, _vp]),
    "rac_rotate_batch_async": (_i, [_vp, _vp, _vp, _ll, _i, _i, _vp]),
    "rac_project_batch_async": (_i, [_vp, _vp, _vp, _ll, _i, _vp]),
    "rac_sincos_batch_async": (_i, [_vp, _vp, _vp, _ll, _vp]),
    "rac_unary_async": (_i, [_vp, _vp, _ll, _i, _vp]),
    "rac_softmax_async": (_i, [_vp, _vp, _ll, _i, _vp]),
    "rac_rmsnorm_async": (_i, [_vp, _vp, _vp, _f, _ll, _i, _vp]),
    "rac_layernorm_async": (_i, [_vp, _vp, _vp, _vp, _f, _ll, _i, _vp]),
    "rac_rope_cache_async": (_i, [_vp, _vp, _i, _i, _f, _vp]),
    "rac_rope_apply_async": (_i, [_vp, _vp, _vp, _vp, _ll, _i, _i, _i, _vp]),
    "rac_check_device_errors": (_i, [_vp]),
    "rac_attention": (None, [_vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i]),
    "rac_attention_async": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _vp]),
}


def exported_symbols() -> list[str]:
    """Names this binding declares (every one must be exported by the .so)."""
    return sorted(_SIGS)


def lib() -> C.CDLL:
    """Loads librac_b200.so once; raises RacError when it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RacError(-4, f"{LIB_PATH} is not built (python -m rac_b200.build)")
                L = C.CDLL(LIB_PATH, mode=os.RTLD_LOCAL | os.RTLD_NOW)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(status: int | None = None) -> None:
    """Raises RacError if `status` (or, when None, rac_last_error()) is non-zero."""
    L = lib()
    st = L.rac_last_error() if status is None else status
    if st != RAC_OK:
        raise RacError(st, L.rac_last_error_string().decode())


CALLS = {"n": 0}     # entry-point calls made through call(); the bench reports it


def call(name: str, *args) -> None:
    """Calls an int-returning entry point and raises on a non-zero status."""
    CALLS["n"] += 1
    check(getattr(lib(), name)(*args))
