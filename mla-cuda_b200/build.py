"""Builds libmla_b200.so (the C-ABI library) in-tree for sm_100a.

Each CUDA source under csrc/ is compiled by nvcc into _build/*.o and linked
into mla-cuda_b200/lib/libmla_b200.so. Objects are rebuilt when their source
or any header under csrc/ or include/ is newer. Usage:

    python mla-cuda_b200/build.py [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libmla_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE), "-I", str(CSRC),
] + ARCH
if os.environ.get("MLA_TC_PROFILE"):        # debug: per-wait cycle accounting in the tensor-core kernel
    NVCC_FLAGS.append("-DMLA_TC_PROFILE")
NVCC_FLAGS += os.environ.get("NVCC_EXTRA", "").split()     # debug / tuning defines


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _newest_header() -> float:
    stamps = [p.stat().st_mtime for d in (CSRC, INCLUDE) for p in d.glob("*.cuh")]
    stamps += [p.stat().st_mtime for p in INCLUDE.glob("*.h")]
    stamps.append(Path(__file__).stat().st_mtime)
    return max(stamps)


def _compile(src: Path, force: bool, hdr: float, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr):
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr = _newest_header()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hdr, extra), srcs))
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), "-shared", *ARCH, "-o", str(LIB), *map(str, objs), "-lcudart", "-lcuda"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage")
    args = ap.parse_args()
    print(build(args.force, args.jobs, args.ptxas_v))
    sys.exit(0)
