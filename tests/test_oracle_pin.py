"""Pins the CPU oracle (oracle/oracle.c) before it is trusted as the checker:
against the reference's own known-answer tests (restated in tests/golden/),
against outputs of the reference's own compiled CPU code recorded in
tests/golden/oracle_pin.npz, and — where oracle/_ref was built from the
reference sources — against that library directly, bit for bit."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

from oracle import oracle as O

INVALID = 0xFFFFFFFF


def test_half_widening_is_exact():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ours = O.widen(bits.view(np.float16))
    ref = bits.view(np.float16).astype(np.float32)
    same = (ours.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(ours) & np.isnan(ref))
    assert same.all()


def test_kat_head_3x8x17(golden_dir):
    k = json.load(open(os.path.join(golden_dir, "kat_head_3x8x17.json")))
    h = np.array(k["hidden_f16_bits"], np.uint16).view(np.float16).reshape(k["rows"], -1)
    e = np.array(k["embedding_f16_bits"], np.uint16).view(np.float16).reshape(k["vocabulary_size"], -1)
    allowed = np.array(k["allowed"], np.uint32)
    got, best = O.restricted_head_padded(h, e, allowed, np.array(k["counts"], np.uint32),
                                         k["maximum_allowed"])
    assert got.tolist() == k["expected"]
    assert np.isnan(best[2])


def test_kat_invalid_rows(golden_dir):
    k = json.load(open(os.path.join(golden_dir, "kat_invalid_rows.json")))
    h = np.zeros((k["rows"], k["hidden_size"]), np.float16)
    e = np.zeros((k["vocabulary_size"], k["hidden_size"]), np.float16)
    got, _ = O.restricted_head_padded(h, e, np.array(k["allowed"], np.uint32),
                                      np.array(k["counts"], np.uint32), k["maximum_allowed"])
    assert got.tolist() == k["expected"]


def test_kat_greedy(golden_dir):
    sys.path.insert(0, golden_dir)
    from make_golden import greedy_case

    for case in json.load(open(os.path.join(golden_dir, "kat_greedy.json")))["cases"]:
        logits, exp = greedy_case(case["rows"], case["vocabulary_size"])
        assert O.greedy_select_f16(logits).tolist() == exp == case["expected"]


def test_kat_restricted_greedy_market_dfa(golden_dir):
    sys.path.insert(0, golden_dir)
    from make_golden import market_dfa_case

    z = np.load(os.path.join(golden_dir, "market_dfa.npz"))
    logits, allowed, counts, expected = market_dfa_case(z["state_offsets"], z["arc_tokens"])
    got = O.restricted_greedy_select_f16(logits, allowed, counts, allowed.shape[1])
    assert np.array_equal(got, expected) and np.array_equal(expected, z["select_expected"])


def test_restricted_greedy_invalid_rows():
    """tests/cuda/cuda_tests.cu:1173-1277 (count 0, count > max, id >= V)."""
    logits = np.zeros((1, 8), np.float16)
    for counts, al in (([0], [1, 3, 5, 7]), ([5], [1, 3, 5, 7]), ([2], [1, 8, 5, 7])):
        got = O.restricted_greedy_select_f16(logits, np.array(al, np.uint32),
                                             np.array(counts, np.uint32), 4)
        assert got[0] == INVALID


def test_pr4_real_logits(golden_dir):
    """Real SmolLM2 logits: the oracle's full argmax gives tokens [198, 198,
    504] with the recorded margins (smollm2-pr4-greedy-f32.json), both on the
    FP32 logits (CpuSmolLm2's argmax, src/cpu/smollm2.cpp:444-462) and after
    fp16 rounding (the GPU selection input)."""
    z = np.load(os.path.join(golden_dir, "pr4_logits.npz"))
    lg = z["logits"]
    assert z["tokens"].tolist() == [198, 198, 504]
    assert lg.argmax(axis=1).tolist() == [198, 198, 504]
    top2 = np.sort(lg, axis=1)[:, -2:]
    np.testing.assert_allclose(top2[:, 1] - top2[:, 0], z["margins"], rtol=1e-6)
    assert O.greedy_select_f16(lg.astype(np.float16)).tolist() == [198, 198, 504]
    # the restricted head over an allowed set that excludes the winner
    allowed = np.array([[5, 198, 900, 17]], np.uint32).repeat(3, 0)
    got = O.restricted_greedy_select_f16(lg.astype(np.float16), allowed, np.full(3, 4, np.uint32), 4)
    assert got[0] == 198


def test_oracle_matches_recorded_reference_outputs(golden_dir):
    """oracle.c vs the reference's compiled linear_f32 / rms_norm_f32
    outputs recorded by tests/golden/make_golden.py (bit-exact)."""
    from market_sim_b200 import synth

    z = np.load(os.path.join(golden_dir, "oracle_pin.npz"))
    seed, rows, vocab, kmax = (int(z[k]) for k in ("seed", "rows", "vocab", "kmax"))
    emb = synth.embedding(seed, vocab=vocab)
    hid = synth.hidden_states(seed, rows)
    off, ids = synth.ragged_batch(seed, rows=rows, kmax=kmax, vocab=vocab)
    logits = O.linear_f32(O.widen(hid), O.widen(emb))
    assert np.array_equal(logits.view(np.uint32), z["logits_bits"])
    got, best, _ = O.restricted_head_csr(hid, emb, off, ids)
    assert np.array_equal(got, z["ref_ids"])
    assert np.array_equal(best.view(np.uint32), z["ref_best_bits"])
    full, fbest = O.full_logits_masked_head_csr(hid, emb, off, ids, threads=3)
    assert np.array_equal(full, got) and np.array_equal(fbest.view(np.uint32), best.view(np.uint32))
    rms = O.rms_norm_f32(z["rms_x"], z["rms_gamma"])
    assert np.array_equal(rms.view(np.uint32), z["rms_out_bits"])


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (needs the reference sources)")
def test_oracle_matches_reference_library_live():
    from market_sim_b200 import synth

    emb = synth.embedding(31, vocab=2048)
    hid = synth.hidden_states(31, 5)
    off, ids = synth.ragged_batch(31, rows=5, kmax=700, vocab=2048)
    a, b, _ = O.restricted_head_csr(hid, emb, off, ids)
    c, d = O.ref_full_logits_masked_head_csr(hid, O.widen(emb), off, ids, threads=2)
    assert np.array_equal(a, c) and np.array_equal(b.view(np.uint32), d.view(np.uint32))
    x = synth.normal(31, 4, 3 * 576).astype(np.float32).reshape(3, 576)
    g = synth.normal(31, 5, 576, 1.0, 0.02).astype(np.float32)
    assert np.array_equal(O.rms_norm_f32(x, g).view(np.uint32), O.ref_rms_norm_f32(x, g).view(np.uint32))


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (needs the reference sources)")
def test_market_dfa_fixture_matches_reference():
    off, tok, nxt, term = O.ref_market_dfa()
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "market_dfa.npz"))
    assert np.array_equal(off, z["state_offsets"]) and np.array_equal(tok, z["arc_tokens"])
    assert np.array_equal(nxt, z["arc_next"]) and np.array_equal(term, z["terminal"])
    # ActionDfa::advance agrees with the CSR arc table
    r = O.ref_lib()
    for s in range(0, len(off) - 1, 97):
        for k in range(off[s], off[s + 1]):
            assert r.mfref_market_dfa_advance(s, int(tok[k])) == nxt[k]
    assert len(off) - 1 == 3230 and len(tok) == 3229 and np.diff(off).max() == 11


def test_dfa_decode_oracle_follows_advance():
    """The oracle's decode walks arcs exactly like TokenDfa::advance."""
    from market_sim_b200 import synth

    off, tok, nxt = synth.synthetic_dfa(3, num_states=8, kmax=64, vocab=512)
    emb = synth.embedding(3, vocab=512)
    hid = synth.decode_hidden(3, 6, 4)
    init = np.arange(4, dtype=np.uint32)
    t1, s1 = O.dfa_decode(hid, emb, off, tok, 8, init)
    t2, s2 = O.dfa_decode(hid, emb, off, tok, 8, init, arc_next=nxt)
    assert np.array_equal(t1, t2) and np.array_equal(s1, s2)
    for s in range(6):
        for b in range(4):
            st = s1[s, b]
            cands = tok[off[st]:off[st + 1]]
            x = O.widen(hid[s, b][None])
            logits = O.linear_f32(x, O.widen(emb[cands]))[0]
            assert t1[s, b] == cands[int(np.argmax(logits))]


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (needs the reference sources)")
def test_reference_vocab_split_mode_is_bit_identical():
    """With fewer rows than threads the reference arm splits each row's
    vocabulary over threads; every logit is still one linear_f32 dot."""
    from market_sim_b200 import synth

    emb = synth.embedding(41, vocab=3000)
    hid = synth.hidden_states(41, 2)
    off, ids = synth.ragged_batch(41, rows=2, kmax=900, vocab=3000)
    a, b, _ = O.restricted_head_csr(hid, emb, off, ids)
    c, d = O.ref_full_logits_masked_head_csr(hid, O.widen(emb), off, ids, threads=7)
    assert np.array_equal(a, c) and np.array_equal(b.view(np.uint32), d.view(np.uint32))
