"""ctypes wrapper of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Loads ``oracle/liboracle.so`` (oracle.c, the C restatement of the
reference's CPU path) and, when it was built, ``oracle/_ref/libmfref.so``
(the reference's own CPU sources).  Only tests/, ``__graft_entry__.smoke``
and bench.py's CPU-baseline / reference legs use this module, and only as a
checker or a timed CPU baseline; the product never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libmfref.so")
REF_GPU_LIB = os.path.join(HERE, "_ref", "libmfref_gpu.so")
INVALID = 0xFFFFFFFF

_P = ctypes.c_void_p
_U64 = ctypes.c_uint64


def reference_root():
    """Where the reference's sources lie: $REF when set, else the
    `reference_path` recorded in the repository's BASELINE.json; None when
    neither names an existing directory (e.g. on a GPU box, which only uses
    the libraries built beforehand)."""
    path = os.environ.get("REF")
    if not path:
        cfg = os.path.join(os.path.dirname(HERE), "BASELINE.json")
        if os.path.exists(cfg):
            import json

            with open(cfg) as f:
                path = json.load(f).get("reference_path")
    return path if path and os.path.isdir(path) else None


def build(ref: bool = False) -> None:
    """Compile the oracle (and the reference CPU library when asked and the
    reference sources are present)."""
    targets = ["all"]
    root = reference_root() if ref else None
    if root:
        targets += ["ref", f"REF={root}"]
    subprocess.run(["make", "-s", "-C", HERE, *targets], check=True)


def _load():
    if not os.path.exists(LIB):
        build()
    lib = ctypes.CDLL(LIB)
    lib.orc_half_to_float.argtypes = [ctypes.c_uint16]
    lib.orc_half_to_float.restype = ctypes.c_float
    lib.orc_splitmix64.argtypes = [_U64]
    lib.orc_splitmix64.restype = _U64
    lib.orc_dfa_next.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
    lib.orc_dfa_next.restype = ctypes.c_uint32
    for name, args in {
        "orc_half_to_float_array": [_P, _P, _U64],
        "orc_rms_norm_f32": [_P, _P, _U64, _U64, ctypes.c_float, _P],
        "orc_linear_f32": [_P, _P, _U64, _U64, _U64, _P],
        "orc_restricted_head_csr": [_P, _P, _P, _P, _U64, _U64, _U64, _P, _P, _P, ctypes.c_int],
        "orc_full_logits_masked_head_csr": [_P, _P, _P, _P, _U64, _U64, _U64, _P, _P, ctypes.c_int],
        "orc_greedy_select_f16": [_P, _U64, _U64, _P],
        "orc_restricted_greedy_select_f16": [_P, _P, _P, _U64, _U64, _U64, _P],
        "orc_restricted_head_padded": [_P, _P, _P, _P, _U64, _U64, _U64, _U64, _P, _P],
        "orc_dense_head": [_P, _P, _U64, _U64, _U64, _U64, _P, _P, _P],
        "orc_dfa_decode": [_P, _P, _P, _P, _P, ctypes.c_uint32, _P, _U64, _U64, _U64, _U64, _P, _P],
    }.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = None
    return lib


lib = _load()


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def widen(h: np.ndarray) -> np.ndarray:
    """fp16 -> fp32 by the oracle's own exact conversion."""
    h = np.ascontiguousarray(h, dtype=np.float16)
    out = np.empty(h.shape, dtype=np.float32)
    lib.orc_half_to_float_array(_p(h.view(np.uint16)), _p(out), h.size)
    return out


def rms_norm_f32(x, w, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    rows = x.size // w.size
    lib.orc_rms_norm_f32(_p(x), _p(w), rows, w.size, eps, _p(out))
    return out


def linear_f32(x, w):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty((x.shape[0], w.shape[0]), np.float32)
    lib.orc_linear_f32(_p(x), _p(w), x.shape[0], x.shape[1], w.shape[0], _p(out))
    return out


def restricted_head_csr(hidden_f16, emb_f16, offsets, ids, threads=1):
    """-> (ids u32[rows], best f32[rows], runner_up f32[rows])."""
    hidden = widen(hidden_f16)
    emb = np.ascontiguousarray(emb_f16, np.float16)
    offsets = np.ascontiguousarray(offsets, np.int32)
    ids = np.ascontiguousarray(ids, np.int32)
    rows = hidden.shape[0]
    out = np.empty(rows, np.uint32)
    best = np.empty(rows, np.float32)
    ru = np.empty(rows, np.float32)
    lib.orc_restricted_head_csr(_p(hidden), _p(emb.view(np.uint16)), _p(offsets), _p(ids), rows,
                                hidden.shape[1], emb.shape[0], _p(out), _p(best), _p(ru), threads)
    return out, best, ru


def full_logits_masked_head_csr(hidden_f16, emb_f16, offsets, ids, threads=1):
    hidden = widen(hidden_f16)
    emb = np.ascontiguousarray(emb_f16, np.float16)
    offsets = np.ascontiguousarray(offsets, np.int32)
    ids = np.ascontiguousarray(ids, np.int32)
    rows = hidden.shape[0]
    out = np.empty(rows, np.uint32)
    best = np.empty(rows, np.float32)
    lib.orc_full_logits_masked_head_csr(_p(hidden), _p(emb.view(np.uint16)), _p(offsets), _p(ids),
                                        rows, hidden.shape[1], emb.shape[0], _p(out), _p(best),
                                        threads)
    return out, best


def restricted_head_padded(hidden_f16, emb_f16, allowed, counts, max_allowed):
    hidden = widen(hidden_f16)
    emb = np.ascontiguousarray(emb_f16, np.float16)
    allowed = np.ascontiguousarray(allowed, np.uint32)
    counts = np.ascontiguousarray(counts, np.uint32)
    rows = hidden.shape[0]
    out = np.empty(rows, np.uint32)
    best = np.empty(rows, np.float32)
    lib.orc_restricted_head_padded(_p(hidden), _p(emb.view(np.uint16)), _p(allowed), _p(counts),
                                   rows, hidden.shape[1], emb.shape[0], max_allowed, _p(out),
                                   _p(best))
    return out, best


def greedy_select_f16(logits_f16):
    lg = np.ascontiguousarray(logits_f16, np.float16)
    out = np.empty(lg.shape[0], np.uint32)
    lib.orc_greedy_select_f16(_p(lg.view(np.uint16)), lg.shape[0], lg.shape[1], _p(out))
    return out


def restricted_greedy_select_f16(logits_f16, allowed, counts, max_allowed):
    lg = np.ascontiguousarray(logits_f16, np.float16)
    allowed = np.ascontiguousarray(allowed, np.uint32)
    counts = np.ascontiguousarray(counts, np.uint32)
    out = np.empty(lg.shape[0], np.uint32)
    lib.orc_restricted_greedy_select_f16(_p(lg.view(np.uint16)), _p(allowed), _p(counts),
                                         lg.shape[0], lg.shape[1], max_allowed, _p(out))
    return out


def dense_head(hidden_f16, emb_f16, vocab_begin=0, vocab_end=None):
    hidden = widen(hidden_f16)
    emb = np.ascontiguousarray(emb_f16, np.float16)
    vocab_end = emb.shape[0] if vocab_end is None else vocab_end
    rows = hidden.shape[0]
    out = np.empty(rows, np.uint32)
    best = np.empty(rows, np.float32)
    ru = np.empty(rows, np.float32)
    lib.orc_dense_head(_p(hidden), _p(emb.view(np.uint16)), rows, hidden.shape[1], vocab_begin,
                       vocab_end, _p(out), _p(best), _p(ru))
    return out, best, ru


def dfa_decode(hidden_f16, emb_f16, dfa_offsets, dfa_ids, num_states, init_states, arc_next=None):
    """hidden_f16 [steps, batch, H] -> (tokens [steps, batch], states [steps+1, batch]).
    arc_next None = the synthetic hash transition, else the per-arc table."""
    steps, batch, h = hidden_f16.shape
    hidden = widen(hidden_f16)
    emb = np.ascontiguousarray(emb_f16, np.float16)
    off = np.ascontiguousarray(dfa_offsets, np.int32)
    ids = np.ascontiguousarray(dfa_ids, np.int32)
    init = np.ascontiguousarray(init_states, np.uint32)
    tokens = np.empty((steps, batch), np.uint32)
    states = np.empty((steps + 1, batch), np.uint32)
    nxt = None if arc_next is None else np.ascontiguousarray(arc_next, np.uint32)
    lib.orc_dfa_decode(_p(hidden), _p(emb.view(np.uint16)), _p(off), _p(ids),
                       None if nxt is None else _p(nxt), num_states,
                       _p(init), steps, batch, h, emb.shape[0], _p(tokens), _p(states))
    return tokens, states


# ---- the reference's own CPU code (oracle/_ref), when built --------------

def ref_available() -> bool:
    return os.path.exists(REF_LIB)


_ref = None


def ref_lib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"{REF_LIB} not built (make -C oracle ref)")
        r = ctypes.CDLL(REF_LIB)
        r.mfref_rms_norm_f32.argtypes = [_P, _P, _U64, _U64, ctypes.c_float, _P]
        r.mfref_linear_f32.argtypes = [_P, _P, _U64, _U64, _U64, _P]
        r.mfref_full_logits_masked_head_csr.argtypes = [_P, _P, _P, _P, _U64, _U64, _U64, _P, _P,
                                                        ctypes.c_int]
        r.mfref_head_csr_by_sequence.argtypes = [_P, _P, _P, _P, _U64, _U64, _U64, _P, _P,
                                                 ctypes.c_int]
        r.mfref_market_dfa.argtypes = [_P, _P, _P, _P, _P, _P]
        r.mfref_market_dfa_advance.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        r.mfref_market_dfa_advance.restype = ctypes.c_uint32
        for f in ("mfref_rms_norm_f32", "mfref_linear_f32", "mfref_full_logits_masked_head_csr",
                  "mfref_head_csr_by_sequence", "mfref_market_dfa"):
            getattr(r, f).restype = ctypes.c_int
        _ref = r
    return _ref


def ref_linear_f32(x, w):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty((x.shape[0], w.shape[0]), np.float32)
    code = ref_lib().mfref_linear_f32(_p(x), _p(w), x.shape[0], x.shape[1], w.shape[0], _p(out))
    assert code == 0, code
    return out


def ref_rms_norm_f32(x, w, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    code = ref_lib().mfref_rms_norm_f32(_p(x), _p(w), x.size // w.size, w.size, eps, _p(out))
    assert code == 0, code
    return out


def ref_full_logits_masked_head_csr(hidden_f16, emb_f32, offsets, ids, threads=1):
    hidden = widen(hidden_f16)
    emb_f32 = np.ascontiguousarray(emb_f32, np.float32)
    offsets = np.ascontiguousarray(offsets, np.int32)
    ids = np.ascontiguousarray(ids, np.int32)
    rows = hidden.shape[0]
    out = np.empty(rows, np.uint32)
    best = np.empty(rows, np.float32)
    code = ref_lib().mfref_full_logits_masked_head_csr(
        _p(hidden), _p(emb_f32), _p(offsets), _p(ids), rows, hidden.shape[1], emb_f32.shape[0],
        _p(out), _p(best), threads)
    assert code == 0, code
    return out, best


def ref_head_csr_by_sequence(hidden_f16, emb_f32, offsets, ids, threads=1):
    """The reference CPU path (linear_f32 over every vocab row, masked
    argmax) with the batch's sequences split over `threads` threads of a
    pool that persists between calls.  -> (ids u32[rows], best f32[rows])."""
    hidden = widen(hidden_f16)
    emb_f32 = np.ascontiguousarray(emb_f32, np.float32)
    offsets = np.ascontiguousarray(offsets, np.int32)
    ids = np.ascontiguousarray(ids, np.int32)
    rows = hidden.shape[0]
    out = np.empty(rows, np.uint32)
    best = np.empty(rows, np.float32)
    code = ref_lib().mfref_head_csr_by_sequence(
        _p(hidden), _p(emb_f32), _p(offsets), _p(ids), rows, hidden.shape[1], emb_f32.shape[0],
        _p(out), _p(best), threads)
    assert code == 0, code
    return out, best


def ref_gpu_available() -> bool:
    return os.path.exists(REF_GPU_LIB)


class RefGpuHead:
    """The reference's own CUDA restricted head (oracle/_ref/libmfref_gpu.so:
    marketforge::cuda::restricted_output_head_f16 from src/cuda/greedy.cu,
    through its DeviceBuffer / CudaStream types) on one padded problem.
    Inputs are copied into the reference's own buffers from device tensors;
    run() launches on the reference's stream (stream() gives its handle)."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            r = ctypes.CDLL(REF_GPU_LIB)
            r.mfrefgpu_create.argtypes = [_U64, _U64, _U64, _U64]
            r.mfrefgpu_create.restype = _P
            r.mfrefgpu_upload.argtypes = [_P, ctypes.c_int, _P, _U64]
            r.mfrefgpu_run.argtypes = [_P]
            r.mfrefgpu_stream.argtypes = [_P]
            r.mfrefgpu_stream.restype = _P
            r.mfrefgpu_download.argtypes = [_P, _P]
            r.mfrefgpu_destroy.argtypes = [_P]
            cls._lib = r
        return cls._lib

    def __init__(self, hidden, embedding, allowed, counts, max_allowed):
        """Device tensors: hidden fp16 [rows, H], embedding fp16 [V, H],
        allowed u32/i32 [rows, max_allowed], counts u32/i32 [rows]."""
        rows, h = int(hidden.shape[0]), int(hidden.shape[1])
        self.rows = rows
        self.ctx = self.lib().mfrefgpu_create(rows, h, int(embedding.shape[0]), int(max_allowed))
        if not self.ctx:
            raise RuntimeError("reference CUDA context allocation failed")
        for which, t in enumerate((hidden, embedding, allowed, counts)):
            code = self.lib().mfrefgpu_upload(self.ctx, which, t.data_ptr(),
                                              t.numel() * t.element_size())
            if code:
                raise RuntimeError(f"reference upload {which} failed: {code}")

    def run(self) -> None:
        code = self.lib().mfrefgpu_run(self.ctx)
        if code:
            raise RuntimeError(f"reference restricted_output_head_f16 failed: {code}")

    def stream(self) -> int:
        return int(self.lib().mfrefgpu_stream(self.ctx) or 0)

    def ids(self) -> np.ndarray:
        out = np.empty(self.rows, np.uint32)
        code = self.lib().mfrefgpu_download(self.ctx, _p(out))
        if code:
            raise RuntimeError(f"reference download failed: {code}")
        return out

    def close(self) -> None:
        if self.ctx:
            self.lib().mfrefgpu_destroy(self.ctx)
            self.ctx = None


def ref_market_dfa():
    """The reference's SmolLM2 market-action DFA as CSR numpy arrays."""
    r = ref_lib()
    ns, na = ctypes.c_uint32(), ctypes.c_uint32()
    assert r.mfref_market_dfa(ctypes.byref(ns), ctypes.byref(na), None, None, None, None) == 0
    off = np.empty(ns.value + 1, np.int32)
    tok = np.empty(na.value, np.uint32)
    nxt = np.empty(na.value, np.uint32)
    term = np.empty(ns.value, np.uint8)
    assert r.mfref_market_dfa(ctypes.byref(ns), ctypes.byref(na), _p(off), _p(tok), _p(nxt),
                              _p(term)) == 0
    return off, tok, nxt, term
