"""ctypes binding of ``libmfhead.so`` (the C-ABI in ``include/mf_head.h``).

The library is the product: there is no Python or CPU fallback.  Importing
this module fails loudly when the shared library is missing; build it with
``python -m market_sim_b200.build``.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libmfhead.so")


class MfStatus(ctypes.Structure):
    """``mf_status``: ``code`` uses marketforge::ErrorCode numbering."""

    _fields_ = [("code", ctypes.c_int32), ("detail", ctypes.c_uint32)]


_P = ctypes.c_void_p
_U64 = ctypes.c_uint64

# name -> argument count of (pointer, bytes) pairs and trailing u64 / stream args
_SIGNATURES = {
    "mf_greedy_select_f16": [_P, _U64, _P, _U64, _U64, _U64, _P],
    "mf_restricted_greedy_select_f16": [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _U64, _U64, _U64, _P],
    "mf_restricted_output_head_f16": [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64,
                                      _U64, _U64, _U64, _U64, _P],
    "mf_head_restricted_csr_f16": [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64,
                                   _P, _U64, _U64, _U64, _U64, _P],
    "mf_dfa_head_step_f16": [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64,
                             _P, _U64, _P, _U64, _P, _U64, _U64, _U64, _U64, _U64, _P],
    "mf_dfa_decode_f16": [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64,
                          _P, _U64, _P, _U64, _U64, _U64, _U64, _U64, _U64, _P],
}

_SIGNATURES["mf_head_restricted_csr_f16_ex"] = ([_P, _U64] * 7 + [_U64, _U64, _U64, ctypes.c_uint32,
                                                                     _P])
_SIGNATURES["mf_head_restricted_csr_u16ids_f16_ex"] = _SIGNATURES["mf_head_restricted_csr_f16_ex"]
_SIGNATURES["mf_head_restricted_csr_f16_noalloc"] = [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _P,
                                                     _U64, _P, _U64, _U64, _U64, _U64, _P]

_SIGNATURES["mf_head_restricted_csr_rmsnorm_f16"] = [_P, _U64, _P, _U64, ctypes.c_float, _P, _U64,
                                                     _P, _U64, _P, _U64, _P, _U64, _P, _U64, _P,
                                                     _U64, _U64, _U64, _U64, _P]
_SIGNATURES["mf_dfa_head_step_rmsnorm_f16"] = ([_P, _U64] * 2 + [ctypes.c_float] + [_P, _U64] * 9
                                               + [_U64] * 4 + [_P])
_SIGNATURES["mf_dense_head_f16"] = [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64, _P, _U64,
                                    _U64, _U64, _U64, _U64, _P]
_SIGNATURES["mf_dense_selftest_wait_timeout"] = [_P, ctypes.POINTER(ctypes.c_uint32),
                                                 ctypes.POINTER(ctypes.c_uint32)]
_SIGNATURES["mf_decode_keys"] = [_P, _U64, _P, _U64, _P, _U64, _U64, _P]
_SIGNATURES["mf_exchange_alloc"] = [ctypes.POINTER(_P), _U64, _P]
_SIGNATURES["mf_exchange_free"] = [_P]
_SIGNATURES["mf_exchange_open_peer"] = [_P, ctypes.POINTER(_P)]
_SIGNATURES["mf_exchange_close_peer"] = [_P]
_SIGNATURES["mf_exchange_broken"] = [_P, _P]
_SIGNATURES["mf_dense_head_sharded_f16"] = ([_P, _U64] * 6 + [_U64] * 4
                                            + [_P, _U64, ctypes.c_uint32, ctypes.c_uint32,
                                               ctypes.c_uint32, _P])
_SIGNATURES["mf_dense_head_f16_ex"] = [_P, _U64] * 6 + [_U64] * 4 + [ctypes.c_uint32, _P]

_SIGNATURES["mf_pipeline_create"] = [ctypes.POINTER(_P), _P, _U64, _U64, _U64, _U64, _U64,
                                     ctypes.c_uint32]
_SIGNATURES["mf_pipeline_submit"] = [_P, _P, _U64, _P, _P, _U64, _P, _P, ctypes.POINTER(_U64)]
_SIGNATURES["mf_pipeline_submit_packed"] = [_P, _P, _U64, _U64, _U64, _P, ctypes.POINTER(_U64)]
_SIGNATURES["mf_pipeline_submit_packed_u16ids"] = _SIGNATURES["mf_pipeline_submit_packed"]
_SIGNATURES["mf_pipeline_wait"] = [_P, _U64]
_SIGNATURES["mf_pipeline_synchronize"] = [_P]

_U64_FUNCS = {"mf_head_workspace_bytes": [_U64], "mf_dfa_workspace_bytes": [_U64],
              "mf_dense_workspace_bytes": [_U64], "mf_exchange_bytes": [_U64, ctypes.c_uint32]}
_U32_FUNCS = {"mf_version": [], "mf_built_arch": [], "mf_pipeline_depth": [_P]}
_PTR_FUNCS = {"mf_pipeline_stream": [_P, ctypes.c_uint32]}
_VOID_FUNCS = {"mf_pipeline_destroy": [_P]}

# Optional entry points: bound when the library exports them.
_OPTIONAL: dict[str, list] = {}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library with "
            "`python -m market_sim_b200.build` (no CPU fallback exists)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in _SIGNATURES.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = MfStatus
    for name, args in _U64_FUNCS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = ctypes.c_uint64
    for name, args in _U32_FUNCS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = ctypes.c_uint32
    for name, args in _PTR_FUNCS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = ctypes.c_void_p
    for name, args in _VOID_FUNCS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = None
    for name, args in _OPTIONAL.items():
        f = getattr(lib, name, None)
        if f is not None:
            f.argtypes = args
            f.restype = MfStatus
    return lib


lib = _load()

#: every symbol include/mf_head.h declares (checked by the CPU test suite)
EXPORTED = sorted(list(_SIGNATURES) + list(_U64_FUNCS) + list(_U32_FUNCS) + list(_PTR_FUNCS)
                  + list(_VOID_FUNCS))
