"""Builds the C++ torch extension ``mla_custom_cuda._C`` in place, over the
C-ABI library ``lib/libmla_b200.so`` (built first by build.py), the way the
reference builds its ``mla_custom_cuda`` extension (setup.py:20-26 there).

    python mla-cuda_b200/setup.py build_ext --inplace
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
os.chdir(PKG)
sys.path.insert(0, str(PKG))

import build as libbuild  # noqa: E402

libbuild.build()

setup(
    name="mla_custom_cuda",
    ext_modules=[
        CppExtension(
            name="mla_custom_cuda._C",
            sources=["mla_custom_cuda/csrc/ext.cpp"],
            include_dirs=[str(ROOT / "include"), os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")],
            library_dirs=[str(PKG / "lib")],
            libraries=["mla_b200"],
            extra_compile_args=["-O2"],
            extra_link_args=["-Wl,-rpath,$ORIGIN/../lib"],
        )
    ],
    cmdclass={"build_ext": BuildExtension},
    script_args=sys.argv[1:] or ["build_ext", "--inplace"],
)
