"""Builds the CUDA library in-tree for sm_100a.

``python -m market_sim_b200.build`` compiles every ``csrc/*.cu`` into
``market_sim_b200/libmfhead.so`` (C-ABI declared in ``include/mf_head.h``)
and the C++ ``marketforge::cuda`` wrapper into ``libmarketforge_b200.so``.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libmfhead.so")
CXX_LIB = os.path.join(PKG, "libmarketforge_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile libmfhead.so (and the C++ wrapper) if any source is newer."""
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))
    if force or _stale(LIB, cu + hdr):
        cmd = [_nvcc(), *NVCC_FLAGS, "-shared", "-I", INCLUDE, "-o", LIB, *cu]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
    cpp = sorted(glob.glob(os.path.join(CSRC, "marketforge", "*.cpp")))
    cpp_hdr = sorted(glob.glob(os.path.join(INCLUDE, "marketforge", "**", "*.hpp"), recursive=True))
    if cpp and (force or _stale(CXX_LIB, cpp + cpp_hdr + [LIB])):
        cuda_root = os.path.dirname(os.path.dirname(_nvcc_path()))
        _run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra",
              "-I", INCLUDE, "-I", os.path.join(cuda_root, "include"), "-o", CXX_LIB, *cpp,
              "-L", PKG, "-lmfhead", "-L", os.path.join(cuda_root, "lib64"), "-lcudart",
              "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + os.path.join(cuda_root, "lib64")])
    return LIB


def _nvcc_path() -> str:
    n = _nvcc()
    if os.path.sep in n:
        return n
    from shutil import which
    return which(n) or "/usr/local/cuda/bin/nvcc"


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
