"""Seeded synthetic inputs for the restricted head (host-side, numpy).

Every value comes from a counter-based splitmix64 stream, so the CUDA path,
the CPU oracle and the benchmark see identical bits for a given seed.
Normals use Box-Muller in float64 and are rounded to float32, then float16.
The reference has no dataset for this path: its own benchmark builds
patterned inputs (src/tools/cuda_restricted_output_head_bench.cu:129-140,
250-258); the shapes and distributions here are the ones the benchmark
configurations name (SmolLM2-135M: hidden 576, vocabulary 49,152).
"""
from __future__ import annotations

import numpy as np

HIDDEN = 576
VOCAB = 49_152
RMS_EPS = 1e-5

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
_G = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)


def splitmix64(x: np.ndarray) -> np.ndarray:
    """The splitmix64 output function of x + golden gamma (wrapping u64)."""
    with np.errstate(over="ignore"):
        z = np.asarray(x, dtype=np.uint64) + _G
        z = (z ^ (z >> np.uint64(30))) * _C1
        z = (z ^ (z >> np.uint64(27))) * _C2
        return z ^ (z >> np.uint64(31))


def stream_u64(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """n values of the counter stream (seed, stream)."""
    key = splitmix64(np.uint64((seed * 0x100000001B3 + stream) & 0xFFFFFFFFFFFFFFFF))
    with np.errstate(over="ignore"):
        return splitmix64(key + np.arange(start, start + n, dtype=np.uint64))


def uniform(seed: int, stream: int, n: int) -> np.ndarray:
    """Uniform doubles in (0, 1) from the top 53 bits."""
    u = stream_u64(seed, stream, n) >> np.uint64(11)
    return (u.astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """Box-Muller normals (float64), cos branch only."""
    u1 = uniform(seed, stream, n)
    u2 = uniform(seed, stream + 0x5151, n)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return mean + std * z


def embedding(seed: int, vocab: int = VOCAB, hidden: int = HIDDEN, std: float = 0.02) -> np.ndarray:
    """Tied embedding ~N(0, std) stored fp16 [vocab, hidden]."""
    return normal(seed, 1, vocab * hidden, 0.0, std).astype(np.float32).astype(
        np.float16).reshape(vocab, hidden)


def rms_norm_f32(x: np.ndarray, gamma: np.ndarray, eps: float = RMS_EPS) -> np.ndarray:
    """RMSNorm in float32 (rms_norm_f32's formula, src/cpu/operators.cpp:522-535)."""
    x = x.astype(np.float32)
    ms = (x * x).sum(axis=-1, dtype=np.float32) / np.float32(x.shape[-1])
    inv = np.float32(1.0) / np.sqrt(ms + np.float32(eps))
    return (x * inv[..., None] * gamma.astype(np.float32)).astype(np.float32)


def hidden_states(seed: int, rows: int, hidden: int = HIDDEN, stream: int = 2) -> np.ndarray:
    """RMSNorm'd hidden rows: x ~ N(0,1), gamma ~ N(1, 0.02); stored fp16."""
    x = normal(seed, stream, rows * hidden).astype(np.float32).reshape(rows, hidden)
    gamma = normal(seed, stream + 1000, hidden, 1.0, 0.02).astype(np.float32)
    return rms_norm_f32(x, gamma).astype(np.float16)


def sample_without_replacement(seed: int, stream: int, k: int, n: int) -> np.ndarray:
    """k distinct ids from [0, n), uniform, in draw order (unsorted)."""
    if k >= n:
        keys = stream_u64(seed, stream, n)
        return np.argsort(keys, kind="stable").astype(np.int32)
    out = np.empty(0, dtype=np.int64)
    start = 0
    while out.size < k:
        m = max(16, 2 * (k - out.size))
        draw = ((stream_u64(seed, stream, m, start) >> np.uint64(32)) * np.uint64(n)) >> np.uint64(32)
        start += m
        cat = np.concatenate([out, draw.astype(np.int64)])
        _, first = np.unique(cat, return_index=True)
        out = cat[np.sort(first)]
    return out[:k].astype(np.int32)


def log_uniform_sizes(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    """floor(exp(U * ln(hi))) clamped to [lo, hi] (log-uniform allowed-set sizes)."""
    u = uniform(seed, stream, n)
    k = np.floor(np.exp(u * np.log(float(hi)))).astype(np.int64)
    return np.clip(k, lo, hi)


def ragged_batch(seed: int, rows: int = 256, kmax: int = 4096, vocab: int = VOCAB,
                 sort_ids: bool = False):
    """CSR allowed sets: per-row size log-uniform in [1, kmax], ids uniform
    without replacement.  Returns (offsets int32[rows+1], ids int32[total])."""
    sizes = log_uniform_sizes(seed, 3, rows, 1, kmax)
    offsets = np.zeros(rows + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(sizes)
    ids = np.empty(int(offsets[-1]), dtype=np.int32)
    for r in range(rows):
        s = sample_without_replacement(seed, 1_000_000 + r, int(sizes[r]), vocab)
        ids[offsets[r]:offsets[r + 1]] = np.sort(s) if sort_ids else s
    return offsets.astype(np.int32), ids


def dfa_next(states: np.ndarray, tokens: np.ndarray, num_states: int) -> np.ndarray:
    """Synthetic transition: splitmix64((state << 32) | token) mod num_states."""
    key = (np.asarray(states, dtype=np.uint64) << np.uint64(32)) | np.asarray(tokens, dtype=np.uint64)
    return (splitmix64(key) % np.uint64(num_states)).astype(np.uint32)


def synthetic_dfa(seed: int, num_states: int = 64, kmax: int = 2048, vocab: int = VOCAB):
    """Token DFA as CSR: state s allows sorted arc_tokens[off[s]:off[s+1]]
    (size log-uniform in [1, kmax]); arc k leads to arc_next[k] =
    splitmix64((s << 32) | token) mod num_states."""
    sizes = log_uniform_sizes(seed, 7, num_states, 1, kmax)
    off = np.zeros(num_states + 1, dtype=np.int64)
    off[1:] = np.cumsum(sizes)
    tokens = np.empty(int(off[-1]), dtype=np.int32)
    states = np.empty(int(off[-1]), dtype=np.uint32)
    for s in range(num_states):
        tokens[off[s]:off[s + 1]] = np.sort(sample_without_replacement(seed, 2_000_000 + s,
                                                                       int(sizes[s]), vocab))
        states[off[s]:off[s + 1]] = s
    nxt = dfa_next(states, tokens.astype(np.uint32), num_states)
    return off.astype(np.int32), tokens, nxt


def decode_hidden(seed: int, steps: int, batch: int, hidden: int = HIDDEN) -> np.ndarray:
    """Per-step RMSNorm'd hidden states, fp16 [steps, batch, hidden]."""
    return hidden_states(seed, steps * batch, hidden, stream=11).reshape(steps, batch, hidden)


def algorithmic_bytes_ragged(offsets: np.ndarray, rows: int, hidden: int = HIDDEN) -> int:
    """Bytes the ragged head must move per launch: each candidate's embedding
    row (hidden*2) and id (4), each hidden row, the offsets, and the outputs
    (id + score)."""
    total = int(offsets[-1])
    return total * (hidden * 2 + 4) + rows * hidden * 2 + (rows + 1) * 4 + rows * 8
