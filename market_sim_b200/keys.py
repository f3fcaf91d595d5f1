"""Host-side packed (score, id) keys — the same encoding the kernels use
(market_sim_b200/csrc/common.cuh): the unsigned order of a key is the
selection rule (highest score, lowest id on ties, NaN below every score,
0 = no candidate, all ones = invalid row).  Used to merge per-shard results
on the host or through a collective, and by the tests."""
from __future__ import annotations

import numpy as np

SIGN_FLIP = np.uint64(1 << 63)
INVALID = 0xFFFFFFFF


def pack(scores, ids) -> np.ndarray:
    """float32 scores, uint32 ids -> uint64 keys."""
    s = np.ascontiguousarray(scores, dtype=np.float32).copy()
    s[s == 0] = 0.0  # -0 ties with +0
    b = s.view(np.uint32).astype(np.uint64)
    neg = (b & np.uint64(0x80000000)) != 0
    ordered = np.where(neg, (~b) & np.uint64(0xFFFFFFFF), b | np.uint64(0x80000000))
    ordered = np.where(np.isnan(s), np.uint64(0), ordered)
    lo = (~np.asarray(ids, dtype=np.uint64)) & np.uint64(0xFFFFFFFF)
    return (ordered << np.uint64(32)) | lo


def unpack(keys):
    """uint64 keys -> (ids uint32, scores float32); sentinel rows -> (INVALID, NaN)."""
    k = np.asarray(keys, dtype=np.uint64)
    valid = (k != 0) & (k != np.uint64(0xFFFFFFFFFFFFFFFF))
    ids = ((~k) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    o = (k >> np.uint64(32)).astype(np.uint64)
    pos = (o & np.uint64(0x80000000)) != 0
    bits = np.where(pos, o & np.uint64(0x7FFFFFFF), (~o) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    sc = bits.view(np.float32).copy()
    sc[o == 0] = np.nan
    ids[~valid] = INVALID
    sc[~valid] = np.nan
    return ids, sc


def to_signed(keys) -> np.ndarray:
    """Keys as int64 whose signed order equals the unsigned key order (for a
    signed MAX all-reduce)."""
    return (np.asarray(keys, dtype=np.uint64) ^ SIGN_FLIP).view(np.int64)


def from_signed(keys_i64) -> np.ndarray:
    return np.asarray(keys_i64, dtype=np.int64).view(np.uint64) ^ SIGN_FLIP
