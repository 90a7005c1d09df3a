"""Blocking rac.h calls on HOST buffers large enough to run in several chunks
(upload, kernel and download of consecutive chunks overlap on three streams).

Work units (vectors, rows, (batch, head) planes) are independent, so the
chunked host path must return exactly the bits of the same call on device
tensors (the stream-ordered path, one launch).  Mixed host / device
arguments take the device ones in place.
"""
import ctypes

import numpy as np
import pytest
import torch

from rac_b200 import _lib, ext

pytestmark = pytest.mark.gpu


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _same(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def test_rotate_and_unary_chunks(cuda):
    L = _lib.lib()
    rng = np.random.default_rng(1)
    n = (1 << 21) + 5                                   # 40 MiB staged -> 5 chunks, ragged tail
    v = rng.standard_normal((n, 2)).astype(np.float32)
    th = rng.uniform(-4, 4, n).astype(np.float32)
    out = np.zeros_like(v)
    L.rac_rotate_batch_n(_p(v), _p(th), _p(out), n, 16)
    _lib.check()
    assert _same(out, ext.rotate_batch(_t(v, cuda), _t(th, cuda), 16).cpu())
    pr = np.zeros(n, np.float32)
    L.rac_project_batch_n(_p(v), _p(th), _p(pr), n, 24)
    _lib.check()
    assert _same(pr, ext.project_batch(_t(v, cuda), _t(th, cuda), 24).cpu())
    x = rng.uniform(-20, 20, 3 * n).astype(np.float32)
    y = np.zeros_like(x)
    L.rac_exp_batch(_p(x), _p(y), x.size)
    _lib.check()
    assert _same(y, ext.exp(_t(x, cuda)).cpu())


def test_rows_chunks_and_mixed_arguments(cuda):
    L = _lib.lib()
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((4099, 1024)) * 3).astype(np.float32)   # 32 MiB staged -> 4 chunks
    g = rng.uniform(0.5, 1.5, 1024).astype(np.float32)
    b = (rng.standard_normal(1024) * 0.1).astype(np.float32)
    y = np.zeros_like(x)
    L.rac_softmax_batch(_p(x), _p(y), *x.shape)
    _lib.check()
    assert _same(y, ext.softmax(_t(x, cuda)).cpu())
    L.rac_rmsnorm(_p(x), _p(y), _p(g), ctypes.c_float(1e-6), *x.shape)
    _lib.check()
    want = ext.rmsnorm(_t(x, cuda), _t(g, cuda), 1e-6).cpu()
    assert _same(y, want)
    gd = _t(g, cuda)                                    # gamma on the device, x and y on the host
    y2 = np.zeros_like(x)
    L.rac_rmsnorm(_p(x), _p(y2), ctypes.c_void_p(gd.data_ptr()), ctypes.c_float(1e-6), *x.shape)
    _lib.check()
    assert _same(y2, want)
    L.rac_layernorm(_p(x), _p(y), _p(g), _p(b), ctypes.c_float(1e-6), *x.shape)
    _lib.check()
    assert _same(y, ext.layernorm(_t(x, cuda), _t(g, cuda), _t(b, cuda), 1e-6).cpu())


def test_rope_and_attention_chunks(cuda):
    L = _lib.lib()
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 16, 1024, 128)).astype(np.float32)   # 32 MiB in place -> 4 chunks
    c, s = ext.rope_cache(1024, 128, 10000.0, device=cuda)
    ch, sh = c.cpu().numpy(), s.cpu().numpy()
    xd = _t(x, cuda)
    ext.rope_apply_(xd, c, s)
    xh = x.copy()
    L.rac_rope_apply(_p(xh), _p(ch), _p(sh), *x.shape)
    _lib.check()
    assert _same(xh, xd.cpu())
    q, k, v = (rng.standard_normal((4, 8, 512, 64)).astype(np.float32) for _ in range(3))
    out = np.zeros_like(q)                                # 16 MiB staged -> 2 chunks of 2 batches
    L.rac_attention(_p(q), _p(k), _p(v), None, 1, _p(out), *q.shape)
    _lib.check()
    assert _same(out, ext.attention(_t(q, cuda), _t(k, cuda), _t(v, cuda), None, True).cpu())
