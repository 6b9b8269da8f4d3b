"""Builds the reference's own CUDA extension, mla_kernels.cu, UNMODIFIED, for
sm_100a into oracle/_ref/ (git-ignored; the built .so travels with the tree to
a GPU box). TEST / MEASUREMENT INFRASTRUCTURE: only bench.py's comparison leg
loads it, to time the reference's GPU kernels on a B200 beside this library.

The source is compiled where it lies (REFERENCE_DIR, default the reference
checkout); nothing is copied. Flags follow the reference's setup.py
(setup.py:4-17) with its sm_80/89/90 targets replaced by sm_100a, and the
module is named mla_ref_cuda so that it cannot shadow the drop-in module.

    REFERENCE_DIR=/path/to/mla-cuda python oracle/build_ref.py
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def build() -> Path:
    # default: a "reference" checkout beside this repository
    ref = Path(os.environ.get("REFERENCE_DIR", str(HERE.parent.parent / "reference")))
    src = ref / "mla_kernels.cu"
    if not src.exists():
        raise FileNotFoundError(f"{src} not found (set REFERENCE_DIR)")
    OUT.mkdir(exist_ok=True)
    from torch.utils.cpp_extension import load
    load(name="mla_ref_cuda", sources=[str(src)], build_directory=str(OUT),
         extra_cflags=["-O3"],
         extra_cuda_cflags=["-O3", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                            "-U__CUDA_NO_HALF2_OPERATORS__", "--expt-relaxed-constexpr", "--expt-extended-lambda",
                            "-gencode=arch=compute_100a,code=sm_100a"],
         verbose=False)
    so = OUT / "mla_ref_cuda.so"
    if not so.exists():
        raise RuntimeError("reference extension did not build")
    return so


if __name__ == "__main__":
    print(build())
    sys.exit(0)
