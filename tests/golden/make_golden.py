"""Generates tests/golden/*.npz from the reference library itself.

The vectors come from the reference's own lib/c (rac_cpu.c and friends),
compiled from its sources by oracle/Makefile into oracle/_ref/librac_ref.so,
and -- for the PyTorch module path -- from the reference rac_torch.py module
imported from the reference checkout and run on CPU torch.  Inputs are
seeded; the shapes are small so the fixtures stay a few hundred KB.

    python tests/golden/make_golden.py [--ref-root /path/to/RAC]
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402


def lib_vectors(out: str) -> None:
    rng = np.random.default_rng(20260301)
    n = 4096
    v = rng.standard_normal((n, 2)).astype(np.float32)
    th = rng.uniform(-np.pi, np.pi, n).astype(np.float32)
    # Edge angles: the wrap and fold boundaries, +-0, multiples of pi/2.
    edges = np.array([0.0, -0.0, np.pi, -np.pi, np.pi / 2, -np.pi / 2, 3.0, -3.0,
                      7.0, -7.0, 100.0, -100.0, 1e-30, -1e-30, 2 * np.pi, 1.5707964],
                     np.float32)
    th[:edges.size] = edges
    d = {"rot_v": v, "rot_theta": th, "rot_batch": O.ref_rotate_batch(v, th)}
    for it in (4, 8, 12, 16, 24):
        d[f"rot_n{it}"] = O.ref_rotate_n_batch(v, th, it)
        d[f"proj_n{it}"] = O.ref_project_n_batch(v, th, it)
    c, s = O.ref_rope_cache(64, 128, 10000.0)
    d["rope_cos"], d["rope_sin"] = c, s
    c2, s2 = O.ref_rope_cache(4096, 128, 10000.0)
    pick = np.array([0, 1, 2, 17, 1000, 2047, 4095])
    d["rope4096_rows"], d["rope4096_cos"], d["rope4096_sin"] = pick, c2[pick], s2[pick]
    x = rng.standard_normal((1, 2, 64, 128)).astype(np.float32)
    d["rope_x"], d["rope_out"] = x, O.ref_rope_apply(x, c, s)
    xs = (rng.standard_normal((9, 1000)) * 3).astype(np.float32)
    d["softmax_x"], d["softmax_out"] = xs, O.ref_softmax(xs)
    xn = rng.standard_normal((5, 4096)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, 4096).astype(np.float32)
    b = (rng.standard_normal(4096) * 0.1).astype(np.float32)
    d["norm_x"], d["norm_g"], d["norm_b"] = xn, g, b
    d["rms_out"] = O.ref_rmsnorm(xn, g, 1e-6)
    d["ln_out"] = O.ref_layernorm(xn, g, b, 1e-6)
    xe = np.concatenate([rng.uniform(-20, 20, 2000), [0.0, -0.0, 1.0, -1.0, 88.0, -87.0]]).astype(np.float32)
    L = O.ref()
    d["unary_x"] = xe
    d["exp_out"] = np.array([L.rac_exp(float(t)) for t in xe], np.float32)
    d["tanh_out"] = np.array([L.rac_tanh(float(t)) for t in xe], np.float32)
    xr = np.concatenate([rng.uniform(0, 100, 500), [0.0, -1.0, 4.0, 1e-30]]).astype(np.float32)
    d["rsqrt_x"], d["rsqrt_out"] = xr, np.array([L.rac_rsqrt(float(t)) for t in xr], np.float32)
    A = rng.uniform(-1, 1, (48, 96)).astype(np.float32)
    B = rng.uniform(-1, 1, (96, 40)).astype(np.float32)
    d["mm_A"], d["mm_B"] = A, B
    for it in (8, 16, 24):
        d[f"mm_cordic{it}"] = O.gemm_composed_ref(A, B, it)
    d["mm_sgemm"] = O.ref_sgemm(A, B)
    qa, ka, va = [rng.standard_normal((1, 2, 70, 64)).astype(np.float32) for _ in range(3)]
    am = (rng.standard_normal((70, 70)) * 0.5).astype(np.float32)
    d["att_q"], d["att_k"], d["att_v"], d["att_mask"] = qa, ka, va, am
    d["att_causal"] = O.ref_attention(qa, ka, va, None, True)
    d["att_masked"] = O.ref_attention(qa, ka, va, am, False)
    np.savez_compressed(out, **d)


def module_vectors(out: str, ref_root: str) -> None:
    """Outputs of the reference rac_torch modules on CPU torch (fallback path)."""
    import torch
    sys.path.insert(0, os.path.join(ref_root, "rac_torch"))
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        import rac_torch as R  # the reference module, imported from its checkout
    torch.manual_seed(1234)
    d, H, ff, T, Bt = 64, 4, 160, 24, 2
    blk = R.RACLlamaBlock(d, H, ff_dim=ff, max_seq_len=64, activation="silu", bias=False)
    with torch.no_grad():
        for p in blk.parameters():
            p.copy_(torch.randn_like(p) * 0.02 if p.dim() > 1 else 1.0 + 0.1 * torch.randn_like(p))
    x = torch.randn(Bt, T, d)
    with torch.no_grad():
        y = blk(x, is_causal=True)
        y_nc = blk(x, is_causal=False)
        n1 = blk.norm1(x)
        q = torch.randn(Bt, H, T, d // H)
        k = torch.randn(Bt, H, T, d // H)
        rq, rk = blk.attn.rope(q, k)
    sd = {f"w.{k_}": v.numpy() for k_, v in blk.state_dict().items()}
    np.savez_compressed(out, x=x.numpy(), y=y.numpy(), y_noncausal=y_nc.numpy(),
                        norm1=n1.numpy(), rope_q=q.numpy(), rope_k=k.numpy(),
                        rope_q_out=rq.numpy(), rope_k_out=rk.numpy(),
                        cfg=np.array([d, H, ff, T, Bt, 64]), **sd)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=None,
                    help="reference checkout (default: RAC_REF_ROOT, else ../reference beside the repo)")
    a = ap.parse_args()
    O.build()
    lib_vectors(os.path.join(HERE, "lib_c_vectors.npz"))
    from oracle.build_ref_hip import default_root
    module_vectors(os.path.join(HERE, "rac_torch_block.npz"), a.ref_root or default_root())
    print("wrote", os.listdir(HERE))
