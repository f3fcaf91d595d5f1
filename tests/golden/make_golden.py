"""Generates the golden fixtures in tests/golden/ (run in a container that
has the reference checkout; the GPU box only reads the committed output).

    python tests/golden/make_golden.py [--ref /path/to/reference]

Fixtures and where they come from (paths inside the reference project):
  kat_head_3x8x17.json   tests/cuda/cuda_tests.cu:699-800 — the fused head's
                         3 x 8 x 17 known-answer case (tie between embedding
                         rows 4 and 6, all-NaN hidden row); inputs restated
                         from the test's formulas, expected ids from an exact
                         host FMA loop as the test does.
  kat_invalid_rows.json  tests/cuda/cuda_tests.cu:1341-1404 — count 0,
                         count > max and id >= V rows all give the sentinel.
  kat_greedy.json        tests/cuda/cuda_tests.cu:508-565,1132-1135 — greedy
                         tie/NaN case at V = 17 and V = 49,152 (formula +
                         expected ids).
  market_dfa.npz         the reference's SmolLM2 market-action DFA
                         (SmolLm2MarketActionCatalog::create), dumped through
                         oracle/_ref, plus the restricted-greedy DFA case of
                         tests/cuda/cuda_tests.cu:567-697 (expected ids).
  pr4_logits.npz         tests/fixtures/golden/smollm2-pr4-greedy-f32.safetensors
                         — real SmolLM2 logits [3, 49152], tokens, margins.
  oracle_pin.npz         outputs of the reference's own compiled CPU code
                         (oracle/_ref: linear_f32, rms_norm_f32) on seeded
                         inputs from market_sim_b200.synth, to pin
                         oracle/oracle.c bit for bit where _ref is not built.
"""
from __future__ import annotations

import argparse
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

INVALID = 0xFFFFFFFF


def f16_bits(a) -> list:
    return np.asarray(a, dtype=np.float16).view(np.uint16).astype(int).tolist()


def kat_head():
    rows, hidden, vocab, max_allowed = 3, 8, 17, 5
    h = np.array([((i % 11) - 5) / 8.0 for i in range(rows * hidden)], np.float32)
    e = np.array([(((i * 7) % 19) - 9) / 16.0 for i in range(vocab * hidden)], np.float32)
    h = h.astype(np.float16).reshape(rows, hidden)
    e = e.astype(np.float16).reshape(vocab, hidden)
    e[6] = e[4]
    h[2, :] = np.float16(np.nan)
    allowed = np.array([9, 3, 14, 0, 0, 6, 4, 8, 0, 0, 7, 1, 0, 0, 0], np.uint32)
    counts = np.array([3, 3, 2], np.uint32)
    expected = []
    for r in range(rows):
        best, winner, fallback = -np.inf, INVALID, INVALID
        for k in range(counts[r]):
            t = int(allowed[r * max_allowed + k])
            fallback = min(fallback, t)
            s = 0.0  # every product and partial sum here is exact in fp32
            for f in range(hidden):
                s = float(np.float32(float(h[r, f]) * float(e[t, f]) + s))
            if s > best or (s == best and t < winner):
                best, winner = s, t
        expected.append(winner if winner != INVALID else fallback)
    return {
        "source": "tests/cuda/cuda_tests.cu:699-800",
        "rows": rows, "hidden_size": hidden, "vocabulary_size": vocab,
        "maximum_allowed": max_allowed,
        "hidden_f16_bits": f16_bits(h.reshape(-1)), "embedding_f16_bits": f16_bits(e.reshape(-1)),
        "allowed": allowed.tolist(), "counts": counts.tolist(), "expected": expected,
    }


def kat_invalid_rows():
    return {
        "source": "tests/cuda/cuda_tests.cu:1341-1404",
        "rows": 3, "hidden_size": 2, "vocabulary_size": 5, "maximum_allowed": 2,
        "allowed": [1, 2, 2, 3, 1, 5], "counts": [0, 3, 2],
        "expected": [INVALID, INVALID, INVALID],
    }


def greedy_case(rows: int, vocab: int):
    """tests/cuda/cuda_tests.cu:508-533 restated."""
    logits = np.full((rows, vocab), -4.0, np.float16)
    expected = []
    for r in range(rows):
        w = (r * 7 + 3) % vocab
        expected.append(w)
        logits[r, w] = 8.0
    if rows > 1 and vocab > 9:
        logits[1, 9] = 8.0
        expected[1] = 9
    if rows > 2 and vocab > 1:
        logits[2, :] = -np.inf
        logits[2, 0] = np.nan
        expected[2] = 1
    return logits, expected


def kat_greedy():
    cases = []
    for rows, vocab in ((1, 17), (3, 49_152)):
        _, exp = greedy_case(rows, vocab)
        cases.append({"rows": rows, "vocabulary_size": vocab, "expected": exp})
    return {"source": "tests/cuda/cuda_tests.cu:508-565,1132-1135", "cases": cases}


def market_dfa_case(off, tok):
    """tests/cuda/cuda_tests.cu:567-639: first 8 non-empty states, padded
    table, disallowed logit 100 must lose, row 0 ties, row 1 all NaN."""
    vocab = 49_152
    rows_tokens = []
    for s in range(len(off) - 1):
        if len(rows_tokens) == 8:
            break
        t = tok[off[s]:off[s + 1]]
        if t.size:
            rows_tokens.append([int(x) for x in t])
    rows = len(rows_tokens)
    max_allowed = max(len(t) for t in rows_tokens)
    logits = np.full((rows, vocab), -8.0, np.float16)
    allowed = np.full((rows, max_allowed), INVALID, np.uint32)
    counts = np.zeros(rows, np.uint32)
    expected = []
    for r, cands in enumerate(rows_tokens):
        counts[r] = len(cands)
        dis = vocab - 1
        while dis in cands:
            dis -= 1
        logits[r, dis] = 100.0
        best, winner, fallback = -np.inf, INVALID, INVALID
        for i, t in enumerate(cands):
            allowed[r, i] = t
            v = 4.0 if r == 0 else (np.nan if r == 1 else float((t * 17 + r) % 31))
            logits[r, t] = v
            rv = float(logits[r, t])
            fallback = min(fallback, t)
            if rv > best or (rv == best and t < winner):
                best, winner = rv, t
        expected.append(winner if winner != INVALID else fallback)
    return logits, allowed, counts, np.array(expected, np.uint32)


def read_safetensors(path):
    b = open(path, "rb").read()
    n = struct.unpack("<Q", b[:8])[0]
    hdr = json.loads(b[8:8 + n])
    data = b[8 + n:]
    out = {}
    for k, v in hdr.items():
        if k == "__metadata__":
            continue
        dt = {"F32": np.float32, "I32": np.int32}[v["dtype"]]
        s, e = v["data_offsets"]
        out[k] = np.frombuffer(data[s:e], dtype=dt).reshape(v["shape"]).copy()
    return out


def oracle_pin():
    from market_sim_b200 import synth
    from oracle import oracle as O

    seed, rows, vocab = 777, 6, 4096
    emb = synth.embedding(seed, vocab=vocab)
    hid = synth.hidden_states(seed, rows)
    off, ids = synth.ragged_batch(seed, rows=rows, kmax=512, vocab=vocab)
    ref_ids, ref_best = O.ref_full_logits_masked_head_csr(hid, O.widen(emb), off, ids, threads=1)
    logits = O.ref_linear_f32(O.widen(hid), O.widen(emb))
    x = synth.normal(seed, 9, 2 * 576).astype(np.float32).reshape(2, 576)
    g = synth.normal(seed, 10, 576, 1.0, 0.02).astype(np.float32)
    rms = O.ref_rms_norm_f32(x, g)
    return dict(seed=seed, rows=rows, vocab=vocab, kmax=512, ref_ids=ref_ids,
                ref_best_bits=ref_best.view(np.uint32),
                logits_bits=logits.view(np.uint32),
                rms_x=x, rms_gamma=g, rms_out_bits=rms.view(np.uint32))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None,
                    help="the reference project's root (default: $REF, else BASELINE.json's "
                         "reference_path)")
    a = ap.parse_args()
    from oracle import oracle as O

    if a.ref is None:
        a.ref = O.reference_root()
    if a.ref is None:
        ap.error("the reference sources are needed: pass --ref or set REF")
    os.environ["REF"] = a.ref

    O.build(ref=True)
    with open(os.path.join(HERE, "kat_head_3x8x17.json"), "w") as f:
        json.dump(kat_head(), f)
    with open(os.path.join(HERE, "kat_invalid_rows.json"), "w") as f:
        json.dump(kat_invalid_rows(), f)
    with open(os.path.join(HERE, "kat_greedy.json"), "w") as f:
        json.dump(kat_greedy(), f)
    off, tok, nxt, term = O.ref_market_dfa()
    _, allowed, counts, expected = market_dfa_case(off, tok)
    np.savez_compressed(os.path.join(HERE, "market_dfa.npz"), state_offsets=off, arc_tokens=tok,
                        arc_next=nxt, terminal=term, select_allowed=allowed,
                        select_counts=counts, select_expected=expected)
    st = read_safetensors(os.path.join(a.ref, "tests/fixtures/golden/smollm2-pr4-greedy-f32.safetensors"))
    np.savez_compressed(os.path.join(HERE, "pr4_logits.npz"), logits=st["expected.logits"],
                        tokens=st["expected.tokens"], margins=st["expected.margins"])
    np.savez_compressed(os.path.join(HERE, "oracle_pin.npz"), **oracle_pin())
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
