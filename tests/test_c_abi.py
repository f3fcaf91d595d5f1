"""CPU checks of the C-ABI library: it loads, exports every symbol that
include/mf_head.h declares, and rejects bad metadata on the host before any
CUDA call (no GPU is needed for those paths: pointers here are never
dereferenced)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from market_sim_b200 import build

    build.build()
    from market_sim_b200 import _lib

    return _lib


def declared_symbols():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            text = open(os.path.join(ROOT, "include", h)).read()
            names += re.findall(r"^MF_API\s+[\w\s*]+?\b(mf_\w+)\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(lib):
    declared = declared_symbols()
    assert declared, "no MF_API declarations found"
    out = subprocess.run(["nm", "-D", "--defined-only", lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(mf_\w+)$", out, flags=re.M))
    missing = [n for n in declared if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for n in declared:
        assert hasattr(lib.lib, n)
    assert set(lib.EXPORTED) <= set(declared) | set()


def test_built_for_sm100a(lib):
    assert lib.lib.mf_built_arch() == 1000
    assert lib.lib.mf_version() >= 1


def test_workspace_sizes(lib):
    for rows in (1, 7, 256, 10_000):
        b = lib.lib.mf_head_workspace_bytes(rows)
        assert b >= rows * 12 + 16 and b % 16 == 0
        # the DFA decode adds three rotating key buffers of 8 bytes per row
        assert lib.lib.mf_dfa_workspace_bytes(rows) == b + 24 * rows


FAKE = [0x10000 * (i + 1) for i in range(12)]  # distinct, 16-byte aligned, never dereferenced
STREAM = 0xDEAD0


def _p(i):
    return ctypes.c_void_p(FAKE[i])


def test_padded_head_rejections(lib):
    """Validation order of src/cuda/greedy.cu:349-399."""
    from market_sim_b200.head import ErrorCode as E

    f = lib.lib.mf_restricted_output_head_f16
    rows, hs, v, mx = 1, 4, 8, 2

    def call(rows=rows, hs=hs, v=v, mx=mx, stream=STREAM, sizes=None, ptrs=None):
        s = sizes or [rows * hs * 2, v * hs * 2, rows * mx * 4, rows * 4, rows * 4]
        p = ptrs or [_p(0), _p(1), _p(2), _p(3), _p(4)]
        return f(p[0], s[0], p[1], s[1], p[2], s[2], p[3], s[3], p[4], s[4], rows, hs, v, mx,
                 ctypes.c_void_p(stream) if stream else None).code

    assert call(rows=0) == E.invalid_argument
    assert call(mx=0) == E.invalid_argument
    assert call(hs=0) == E.invalid_argument
    assert call(stream=0) == E.invalid_argument
    assert call(rows=2**64 - 1) == E.resource_limit
    assert call(v=2**32) == E.resource_limit
    assert call(mx=2**32) == E.resource_limit
    assert call(hs=2**62, sizes=[0, 0, 8, 4, 4]) == E.arithmetic_overflow
    assert call(sizes=[rows * hs * 2 + 2, v * hs * 2, rows * mx * 4, 4, 4]) == E.invalid_argument
    assert call(ptrs=[_p(0), _p(1), _p(2), _p(3), _p(3)]) == E.invalid_argument
    assert call(ptrs=[_p(0), None, _p(2), _p(3), _p(4)]) == E.invalid_argument


def test_csr_head_rejections(lib):
    from market_sim_b200.head import ErrorCode as E

    f = lib.lib.mf_head_restricted_csr_f16
    rows, hs, v, total = 4, 576, 1000, 10
    ws = lib.lib.mf_head_workspace_bytes(rows)

    def call(rows=rows, hs=hs, v=v, stream=STREAM, sizes=None, ptrs=None, scores=True):
        s = sizes or [rows * hs * 2, v * hs * 2, (rows + 1) * 4, total * 4, rows * 4, rows * 4, ws]
        p = ptrs or [_p(i) for i in range(7)]
        return f(p[0], s[0], p[1], s[1], p[2], s[2], p[3], s[3], p[4], s[4],
                 p[5] if scores else None, s[5] if scores else 0, p[6], s[6], rows, hs, v,
                 ctypes.c_void_p(stream) if stream else None).code

    assert call(rows=0) == E.invalid_argument
    assert call(stream=0) == E.invalid_argument
    assert call(v=2**32) == E.resource_limit
    assert call(rows=2**31) == E.resource_limit
    assert call(sizes=[rows * hs * 2, v * hs * 2, rows * 4, total * 4, rows * 4, rows * 4, ws]) \
        == E.invalid_argument  # offsets must hold rows + 1 entries
    assert call(sizes=[rows * hs * 2, v * hs * 2, (rows + 1) * 4, total * 4 + 2, rows * 4, rows * 4,
                       ws]) == E.invalid_argument
    assert call(sizes=[rows * hs * 2, v * hs * 2, (rows + 1) * 4, total * 4, rows * 4, rows * 4,
                       ws - 16]) == E.invalid_argument  # workspace too small
    assert call(ptrs=[_p(0), _p(1), _p(2), _p(3), _p(4), _p(4), _p(6)]) == E.invalid_argument


def test_dfa_rejections(lib):
    from market_sim_b200.head import ErrorCode as E

    f = lib.lib.mf_dfa_decode_f16
    steps, batch, ns, hs, v, arcs = 3, 4, 5, 576, 1000, 9
    ws = lib.lib.mf_dfa_workspace_bytes(batch)

    def call(steps=steps, batch=batch, ns=ns, sizes=None):
        s = sizes or [steps * batch * hs * 2, v * hs * 2, (ns + 1) * 4, arcs * 4, arcs * 4,
                      (steps + 1) * batch * 4, steps * batch * 4, steps * batch * 4, ws]
        p = [_p(i) for i in range(9)]
        args = []
        for i in range(9):
            args += [p[i], s[i]]
        return f(*args, steps, batch, ns, hs, v, ctypes.c_void_p(STREAM)).code

    assert call(steps=0) == E.invalid_argument
    assert call(batch=0) == E.invalid_argument
    assert call(batch=8193, sizes=[steps * 8193 * hs * 2, v * hs * 2, (ns + 1) * 4, arcs * 4,
                                   arcs * 4, (steps + 1) * 8193 * 4, steps * 8193 * 4,
                                   steps * 8193 * 4, ws]) == E.resource_limit
    assert call(sizes=[steps * batch * hs * 2, v * hs * 2, (ns + 1) * 4, arcs * 4, arcs * 4 - 4,
                       (steps + 1) * batch * 4, steps * batch * 4, steps * batch * 4, ws]) \
        == E.invalid_argument  # arc_next must match arc_tokens


def test_greedy_rejections(lib):
    from market_sim_b200.head import ErrorCode as E

    f = lib.lib.mf_greedy_select_f16
    st = ctypes.c_void_p(STREAM)
    assert f(_p(0), 16, _p(1), 4, 0, 8, st).code == E.invalid_argument
    assert f(_p(0), 16, _p(1), 4, 1, 8, None).code == E.invalid_argument
    assert f(_p(0), 16, _p(1), 4, 1, 7, st).code == E.invalid_argument
    assert f(_p(0), 16, _p(1), 4, 1, 2**32, st).code == E.resource_limit
    assert f(_p(0), 16, _p(0), 4, 1, 8, st).code == E.invalid_argument


def test_dfa_rmsnorm_step_rejections(lib):
    """mf_dfa_head_step_rmsnorm_f16: rms_norm_f32's own checks on eps
    (src/cpu/operators.cpp:498-501), the norm weight's size, alignment and
    aliasing, then the plain step's validation."""
    from market_sim_b200.head import ErrorCode as E

    f = lib.lib.mf_dfa_head_step_rmsnorm_f16
    batch, ns, hs, v, arcs = 4, 5, 576, 1000, 9
    ws = lib.lib.mf_dfa_workspace_bytes(batch)

    def call(eps=1e-5, gamma=1, gamma_bytes=hs * 2, batch=batch, stream=STREAM):
        s = [batch * hs * 2, gamma_bytes, v * hs * 2, (ns + 1) * 4, arcs * 4, arcs * 4,
             batch * 4, batch * 4, batch * 4, batch * 4, ws]
        p = [_p(0), _p(gamma), _p(2), _p(3), _p(4), _p(5), _p(6), _p(7), _p(8), _p(9), _p(10)]
        args = [p[0], s[0], p[1], s[1], ctypes.c_float(eps)]
        for i in range(2, 11):
            args += [p[i], s[i]]
        return f(*args, batch, ns, hs, v, ctypes.c_void_p(stream) if stream else None).code

    assert call(eps=0.0) == E.invalid_argument
    assert call(eps=float("inf")) == E.invalid_argument
    assert call(gamma_bytes=hs * 2 - 2) == E.invalid_argument
    assert call(gamma=0) == E.invalid_argument  # the norm weight aliases the hidden rows
    assert call(batch=0) == E.invalid_argument
    assert call(stream=0) == E.invalid_argument


def test_csr_u16ids_rejections(lib):
    """mf_head_restricted_csr_u16ids_f16_ex: the ids are u16, so a vocabulary
    above 65,536 or an odd byte count is invalid_argument (host checks only)."""
    from market_sim_b200.head import ErrorCode as E

    f = lib.lib.mf_head_restricted_csr_u16ids_f16_ex
    rows, hs, total = 4, 576, 10
    ws = lib.lib.mf_head_workspace_bytes(rows)

    def call(v=1000, ids_bytes=total * 2):
        s = [rows * hs * 2, v * hs * 2, (rows + 1) * 4, ids_bytes, rows * 4, rows * 4, ws]
        p = [_p(i) for i in range(7)]
        args = []
        for i in range(7):
            args += [p[i], s[i]]
        return f(*args, rows, hs, v, 0, ctypes.c_void_p(STREAM)).code

    assert call(v=65537) == E.invalid_argument
    assert call(ids_bytes=total * 2 + 1) == E.invalid_argument


def test_misaligned_buffers_rejected(lib):
    """A buffer that does not start on a multiple of its widest element (2-byte
    halves, 4-byte ints, 8-byte workspace keys) is invalid_argument on the
    host, never a device fault (checked before any CUDA call)."""
    from market_sim_b200.head import ErrorCode as E

    rows, hs, v, total = 4, 576, 1000, 10
    ws = lib.lib.mf_head_workspace_bytes(rows)

    def csr(bump):
        f = lib.lib.mf_head_restricted_csr_f16
        s = [rows * hs * 2, v * hs * 2, (rows + 1) * 4, total * 4, rows * 4, rows * 4, ws]
        p = [ctypes.c_void_p(FAKE[i] + bump.get(i, 0)) for i in range(7)]
        args = []
        for i in range(7):
            args += [p[i], s[i]]
        return f(*args, rows, hs, v, ctypes.c_void_p(STREAM)).code

    assert csr({2: 2}) == E.invalid_argument  # offsets
    assert csr({3: 2}) == E.invalid_argument  # int32 ids
    assert csr({4: 2}) == E.invalid_argument  # out ids
    assert csr({6: 4}) == E.invalid_argument  # workspace (8-byte keys)
    assert csr({0: 1}) == E.invalid_argument  # hidden halves

    f = lib.lib.mf_restricted_output_head_f16
    r, mx = 1, 2
    sz = [r * hs * 2, v * hs * 2, r * mx * 4, r * 4, r * 4]
    p = [ctypes.c_void_p(FAKE[i] + (2 if i == 2 else 0)) for i in range(5)]
    assert f(p[0], sz[0], p[1], sz[1], p[2], sz[2], p[3], sz[3], p[4], sz[4], r, hs, v, mx,
             ctypes.c_void_p(STREAM)).code == E.invalid_argument  # allowed ids

    f = lib.lib.mf_dfa_decode_f16
    steps, batch, ns, arcs = 3, 4, 5, 9
    dws = lib.lib.mf_dfa_workspace_bytes(batch)
    s = [steps * batch * hs * 2, v * hs * 2, (ns + 1) * 4, arcs * 4, arcs * 4,
         (steps + 1) * batch * 4, steps * batch * 4, steps * batch * 4, dws]
    p = [ctypes.c_void_p(FAKE[i] + (2 if i == 3 else 0)) for i in range(9)]
    args = []
    for i in range(9):
        args += [p[i], s[i]]
    assert f(*args, steps, batch, ns, hs, v, ctypes.c_void_p(STREAM)).code == E.invalid_argument


def test_dense_misaligned_outputs_rejected(lib):
    """The dense head and mf_decode_keys reject output buffers that are not
    aligned to their element size (host check, before any CUDA call)."""
    from market_sim_b200.head import ErrorCode as E

    rows, hs, v = 4, 576, 1024
    f = lib.lib.mf_dense_head_f16
    ws = lib.lib.mf_dense_workspace_bytes(rows)
    s = [rows * hs * 2, v * hs * 2, rows * 8, rows * 4, rows * 4, ws]
    p = [ctypes.c_void_p(FAKE[i] + (2 if i == 3 else 0)) for i in range(6)]
    args = []
    for i in range(6):
        args += [p[i], s[i]]
    assert f(*args, rows, hs, v, 0, ctypes.c_void_p(STREAM)).code == E.invalid_argument
    g = lib.lib.mf_decode_keys
    assert g(ctypes.c_void_p(FAKE[0] + 4), rows * 8, _p(1), rows * 4, None, 0, rows,
             ctypes.c_void_p(STREAM)).code == E.invalid_argument
