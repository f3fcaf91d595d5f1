"""Builds the CUDA library in-tree for sm_100a.

``python -m market_sim_b200.build`` compiles every ``csrc/*.cu`` into
``market_sim_b200/libmfhead.so`` (C-ABI declared in ``include/mf_head.h``)
and the C++ ``marketforge::cuda`` wrapper into ``libmarketforge_b200.so``.
"""
from __future__ import annotations

import glob
import hashlib
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


def _digest(deps: list[str], cmd: list[str]) -> str:
    """Hash of the sources' contents and the build command."""
    h = hashlib.sha256()
    # paths inside the tree are hashed relative to it, so a copy of the tree
    # elsewhere keeps the libraries built here
    h.update("\0".join(os.path.relpath(a, ROOT) if a.startswith(ROOT) else a
                        for a in cmd).encode())
    for d in sorted(deps):
        h.update(os.path.relpath(d, ROOT).encode())
        with open(d, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def _stale(target: str, deps: list[str], cmd: list[str]) -> bool:
    """A target is rebuilt unless it exists and the hash recorded beside it
    matches the current sources and command (file times are not trusted: a
    copied tree can carry a library newer than sources it was not built
    from)."""
    stamp = target + ".sha256"
    if not os.path.exists(target) or not os.path.exists(stamp):
        return True
    with open(stamp) as f:
        return f.read().strip() != _digest(deps, cmd)


def _stamp(target: str, deps: list[str], cmd: list[str]) -> None:
    with open(target + ".sha256", "w") as f:
        f.write(_digest(deps, cmd) + "\n")


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile libmfhead.so (and the C++ wrapper) unless the recorded source hash matches."""
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))
    cmd = [_nvcc(), *NVCC_FLAGS, "-shared", "-I", INCLUDE, "-o", LIB, *cu]
    key = [a for a in cmd if a != _nvcc()]
    if force or _stale(LIB, cu + hdr, key):
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
        _stamp(LIB, cu + hdr, key)
    cpp = sorted(glob.glob(os.path.join(CSRC, "marketforge", "*.cpp")))
    cpp_hdr = sorted(glob.glob(os.path.join(INCLUDE, "marketforge", "**", "*.hpp"), recursive=True))
    if cpp:
        cuda_root = os.path.dirname(os.path.dirname(_nvcc_path()))
        cxx = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra",
               "-I", INCLUDE, "-I", os.path.join(cuda_root, "include"), "-o", CXX_LIB, *cpp,
               "-L", PKG, "-lmfhead", "-L", os.path.join(cuda_root, "lib64"), "-lcudart",
               "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + os.path.join(cuda_root, "lib64")]
        deps = cpp + cpp_hdr + [LIB]
        if force or _stale(CXX_LIB, deps, cxx):
            _run(cxx)
            _stamp(CXX_LIB, deps, cxx)
    return LIB


def _nvcc_path() -> str:
    n = _nvcc()
    if os.path.sep in n:
        return n
    from shutil import which
    return which(n) or "/usr/local/cuda/bin/nvcc"


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
