"""The C++ marketforge::cuda interface (include/marketforge/...): a caller
written against the reference's headers compiles and links against
libmarketforge_b200.so here (CPU), and its known-answer tests pass on the
GPU."""
from __future__ import annotations

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "market_sim_b200")
CUDA = "/usr/local/cuda"


def _build(out_dir):
    from market_sim_b200 import build

    build.build()
    exe = os.path.join(out_dir, "head_api_test")
    subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(CUDA, "include"), "-o", exe,
                    os.path.join(ROOT, "tests", "cpp", "head_api_test.cpp"),
                    "-L", PKG, "-lmarketforge_b200", "-lmfhead",
                    "-L", os.path.join(CUDA, "lib64"), "-lcudart",
                    "-Wl,-rpath," + PKG, "-Wl,-rpath," + os.path.join(CUDA, "lib64")],
                   check=True, capture_output=True, text=True)
    return exe


def test_cpp_caller_compiles_and_links(tmp_path):
    exe = _build(str(tmp_path))
    assert os.path.exists(exe)


@pytest.mark.gpu
def test_cpp_caller_known_answers(tmp_path, cuda):
    exe = _build(str(tmp_path))
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ALL PASSED" in r.stdout, r.stdout + r.stderr
