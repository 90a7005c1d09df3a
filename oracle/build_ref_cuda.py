"""Builds the reference's own PyTorch CUDA extension (rac_torch/rac_torch.cu,
module ``rac_cuda_ext``) for sm_100a into ``oracle/_ref/`` -- TEST
INFRASTRUCTURE ONLY: it serves as a parity check and a same-GPU speed
reference for the FAST-mode GEMM, never as part of the product.

The sources are compiled where they lie in the reference tree (nothing is
copied); the flags are the reference's setup.py ones (-O3, --use_fast_math)
with its gencode list replaced by sm_100a.  Without the reference tree the
build is skipped.

    python -m oracle.build_ref_cuda [REFERENCE_ROOT]
"""
from __future__ import annotations

import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def build(ref_root: str | None = None, verbose: bool = False) -> str | None:
    from .build_ref_hip import default_root
    src = os.path.join(ref_root or default_root(), "rac_torch", "rac_torch.cu")
    if not os.path.exists(src):
        return None
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load
    bdir = os.path.join(OUT, "rac_cuda_ext_build")
    os.makedirs(bdir, exist_ok=True)
    mod = load(name="rac_cuda_ext", sources=[src], build_directory=bdir,
               extra_cflags=["-O3", "-std=c++17"],
               extra_cuda_cflags=["-O3", "--use_fast_math",
                                  "-gencode", "arch=compute_100a,code=sm_100a"],
               verbose=verbose)
    so = mod.__file__
    dst = os.path.join(OUT, "rac_cuda_ext.so")
    shutil.copyfile(so, dst)
    return dst


if __name__ == "__main__":
    print(build(*(sys.argv[1:2] or []), verbose=True))
