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


def _build_head_tail(out_dir):
    from market_sim_b200 import build

    build.build()
    exe = os.path.join(out_dir, "smollm2_head_test")
    subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(CUDA, "include"), "-o", exe,
                    os.path.join(ROOT, "tests", "cpp", "smollm2_head_test.cpp"),
                    "-L", PKG, "-lmarketforge_b200", "-lmfhead",
                    "-L", os.path.join(CUDA, "lib64"), "-lcudart",
                    "-Wl,-rpath," + PKG, "-Wl,-rpath," + os.path.join(CUDA, "lib64")],
                   check=True, capture_output=True, text=True)
    return exe


def test_model_tail_overlay_compiles_and_links(tmp_path):
    """SmolLm2OutputHead (the tail of CudaSmolLm2::forward) and a caller of
    it build and link against libmarketforge_b200.so without a GPU."""
    assert os.path.exists(_build_head_tail(str(tmp_path)))


def test_model_tail_overlay_compiles_against_reference_headers(tmp_path):
    """The overlay's source compiles with the reference's own
    include/marketforge headers first on the include path (its DeviceBuffer,
    StreamHandle, Status and Result), so it drops into the reference's
    build unchanged."""
    from oracle import oracle as O

    ref = O.reference_root()
    if ref is None:
        pytest.skip("reference sources not present")
    subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-Wall",
                    "-I", os.path.join(ref, "include"), "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(CUDA, "include"),
                    os.path.join(PKG, "csrc", "marketforge", "smollm2_head.cpp")],
                   check=True, capture_output=True, text=True)


@pytest.mark.gpu
def test_model_tail_overlay_vs_oracle(tmp_path, cuda):
    """The tail on synthetic decoder outputs (3 rows; the last one is
    decoded, read in place): restricted decode over 300 device ids (past the
    reference's 128-id cap), full-vocabulary decode, and 3 grammar tokens over
    a device-resident 64-state DFA, against the FP32 oracle (rms_norm_f32,
    rounded to fp16 as rms_norm_f16 stores it, then the head)."""
    import numpy as np

    from market_sim_b200 import synth
    from oracle import oracle as O

    from helpers import MARGIN

    exe = _build_head_tail(str(tmp_path))
    H, V, rows, steps = 576, 49_152, 3, 3
    emb = synth.embedding(31337)
    hidden = (synth.normal(31338, 1, steps * rows * H) * 3).astype(np.float32).astype(
        np.float16).reshape(steps, rows, H)
    gamma = synth.normal(31339, 2, H, 1.0, 0.02).astype(np.float32).astype(np.float16)
    allowed = synth.sample_without_replacement(31340, 3, 300, V)
    off, tok, nxt = synth.synthetic_dfa(31341, num_states=64, kmax=2048)
    init = np.uint32(5)
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as f:
        f.write(np.array([H, V, rows, allowed.size, len(off) - 1, tok.size, steps],
                         np.uint64).tobytes())
        for a in (hidden, gamma, emb, allowed.astype(np.int32), off.astype(np.int32),
                  tok.astype(np.int32), nxt.astype(np.int32), np.array([init], np.uint32)):
            f.write(np.ascontiguousarray(a).tobytes())
    outp = tmp_path / "out.bin"
    r = subprocess.run([exe, str(inp), str(outp)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "SMOLLM2 HEAD OK" in r.stdout, (r.returncode, r.stdout, r.stderr)
    got = np.fromfile(outp, np.uint32)
    g_restricted, g_greedy = int(got[0]), int(got[1])
    g_tokens, g_states = got[2:2 + steps], got[2 + steps:2 + 2 * steps]

    def normed(k):
        x = O.widen(hidden[k, rows - 1][None])
        return O.rms_norm_f32(x, O.widen(gamma), 1e-5).astype(np.float16)

    def pick(h16, ids):
        off2 = np.array([0, ids.size], np.int32)
        oid, best, ru = O.restricted_head_csr(h16, emb, off2, ids.astype(np.int32))
        return int(oid[0]), float(best[0] - ru[0])

    oid, margin = pick(normed(0), allowed)
    assert g_restricted == oid or margin < MARGIN
    oid, margin = pick(normed(0), np.arange(V, dtype=np.int32))
    assert g_greedy == oid or margin < MARGIN
    state = int(init)
    for k in range(steps):
        arcs = tok[off[state]:off[state + 1]]
        oid, margin = pick(normed(k), arcs)
        assert int(g_tokens[k]) == oid or margin < MARGIN, (k, g_tokens[k], oid)
        arc = off[state] + int(np.nonzero(arcs == int(g_tokens[k]))[0][0])
        state = int(nxt[arc])
        assert int(g_states[k]) == state
