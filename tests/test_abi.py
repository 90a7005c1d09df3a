"""The C-ABI library: loads, exports every declared entry point, host logic.

No GPU is needed: these tests make no compute calls.  Without a device, a
compute entry point must report RAC_ERR_CUDA rather than fall back to the CPU.
"""
import ctypes
import os
import re

import pytest

from rac_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in ("rac.h", "rac_b200.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(rac_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    missing = [n for n in sorted(_declared()) if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert _declared() == set(_lib.exported_symbols())


def test_no_reference_or_oracle_symbols_in_product():
    out = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    assert "orc_" not in out
    assert "rac_sgemm" not in out and "rac_hal_" not in out


def test_knobs():
    L = _lib.lib()
    L.rac_set_cordic_iters(8)
    assert L.rac_get_cordic_iters() == 8
    L.rac_set_cordic_iters(99)
    assert L.rac_get_cordic_iters() == 24
    L.rac_set_cordic_iters(0)
    assert L.rac_get_cordic_iters() == 16
    L.rac_set_cordic_mode(0)
    assert L.rac_get_cordic_mode() == 0
    L.rac_set_cordic_mode(7)
    assert L.rac_get_cordic_mode() == 0
    L.rac_set_cordic_mode(2)
    assert L.rac_get_cordic_mode() == 2
    L.rac_set_cordic_mode(1)
    assert L.rac_get_cordic_mode() == 1


def test_argument_validation_without_device():
    L = _lib.lib()
    L.rac_matmul(None, None, None, 4, 4, 4)
    assert L.rac_last_error() == -1
    L.rac_rope_cache(None, None, 4, 4, 10000.0)
    assert L.rac_last_error() == -1
    buf = (ctypes.c_float * 8)()
    L.rac_rope_cache(buf, buf, 4, 3, 10000.0)       # odd head_dim
    assert L.rac_last_error() == -2
    L.rac_rotate_batch_n(buf, buf, buf, -1, 16)
    assert L.rac_last_error() == -2
    L.rac_clear_error()
    assert L.rac_last_error() == 0


@pytest.mark.skipif(_lib.lib().rac_b200_device_count() > 0, reason="a device is present")
def test_no_cpu_fallback_without_device():
    L = _lib.lib()
    a = (ctypes.c_float * 16)(*range(16))
    c = (ctypes.c_float * 16)()
    L.rac_matmul(a, a, c, 4, 4, 4)
    assert L.rac_last_error() == -4
    assert list(c) == [0.0] * 16
    assert L.rac_create_context(0) is None


def test_context_rejects_other_backends():
    L = _lib.lib()
    assert L.rac_create_context(2) is None          # RAC_BACKEND_CPU
    assert L.rac_last_error() == -5
