"""GPU parity tests for the restricted head and the selection kernels, all
through the C-ABI (market_sim_b200.head mirrors the reference's
marketforge::cuda functions over it).  The known-answer cases restate the
reference's own CUDA tests (tests/cuda/cuda_tests.cu); the seeded cases
compare against the FP32 CPU oracle (oracle/oracle.c)."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from helpers import INVALID, check_head_parity, gpu_stream, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf(cuda):
    from market_sim_b200 import head

    return head


@pytest.fixture(scope="module")
def O():
    from oracle import oracle

    return oracle


@pytest.fixture(scope="module")
def emb_full(cuda):
    from market_sim_b200 import synth

    e = synth.embedding(20251201)
    return e, to_dev(e)


def _u32(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint32)


def _stream():
    return gpu_stream()


def _csr_call(mf, hidden, emb_dev, offsets, ids, vocab=None, hidden_size=None, ws=None):
    import torch

    rows = int(hidden.shape[0])
    vocab = int(emb_dev.shape[0]) if vocab is None else vocab
    hidden_size = int(hidden.shape[1]) if hidden_size is None else hidden_size
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    if ws is None:
        ws = torch.zeros(mf.head_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    ids_d = to_dev(ids) if ids.size else torch.empty(0, dtype=torch.int32, device="cuda")
    st = mf.restricted_output_head_csr_f16(to_dev(hidden) if isinstance(hidden, np.ndarray) else hidden,
                                           emb_dev, to_dev(offsets), ids_d, out, sc, ws, rows,
                                           hidden_size, vocab, _stream())
    assert st.ok(), st
    torch.cuda.synchronize()
    return _u32(out), sc.cpu().numpy(), ws


# ---- known-answer tests from the reference --------------------------------

def test_kat_head_3x8x17_padded(mf, golden_dir):
    """tests/cuda/cuda_tests.cu:699-800 through restricted_output_head_f16."""
    import torch

    k = json.load(open(os.path.join(golden_dir, "kat_head_3x8x17.json")))
    h = np.array(k["hidden_f16_bits"], np.uint16).view(np.float16)
    e = np.array(k["embedding_f16_bits"], np.uint16).view(np.float16)
    out = torch.empty(k["rows"], dtype=torch.int32, device="cuda")
    st = mf.restricted_output_head_f16(to_dev(h), to_dev(e), to_dev(np.array(k["allowed"], np.uint32)),
                                       to_dev(np.array(k["counts"], np.uint32)), out, k["rows"],
                                       k["hidden_size"], k["vocabulary_size"], k["maximum_allowed"],
                                       _stream())
    assert st.ok(), st
    assert _u32(out).tolist() == k["expected"]


def test_kat_head_3x8x17_csr(mf, golden_dir):
    k = json.load(open(os.path.join(golden_dir, "kat_head_3x8x17.json")))
    h = np.array(k["hidden_f16_bits"], np.uint16).view(np.float16).reshape(k["rows"], -1)
    e = np.array(k["embedding_f16_bits"], np.uint16).view(np.float16).reshape(k["vocabulary_size"], -1)
    allowed = np.array(k["allowed"], np.int32).reshape(k["rows"], -1)
    ids = np.concatenate([allowed[r, :c] for r, c in enumerate(k["counts"])]).astype(np.int32)
    off = np.concatenate([[0], np.cumsum(k["counts"])]).astype(np.int32)
    got, sc, ws = _csr_call(mf, h, to_dev(e), off, ids)
    assert got.tolist() == k["expected"]
    assert np.isnan(sc[2]) and not np.isnan(sc[:2]).any()
    assert int(ws.sum()) == 0, "workspace must be left zero"


def test_kat_invalid_rows_padded(mf, golden_dir):
    """tests/cuda/cuda_tests.cu:1341-1404: count 0, count > max, id >= V."""
    import torch

    k = json.load(open(os.path.join(golden_dir, "kat_invalid_rows.json")))
    rows, hs, v, mx = k["rows"], k["hidden_size"], k["vocabulary_size"], k["maximum_allowed"]
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    st = mf.restricted_output_head_f16(
        torch.zeros(rows * hs, dtype=torch.float16, device="cuda"),
        torch.zeros(v * hs, dtype=torch.float16, device="cuda"),
        to_dev(np.array(k["allowed"], np.uint32)), to_dev(np.array(k["counts"], np.uint32)), out,
        rows, hs, v, mx, _stream())
    assert st.ok()
    assert _u32(out).tolist() == k["expected"]


def test_csr_invalid_rows(mf):
    """CSR counterparts of the invalid-row cases: empty row, id >= V, id < 0."""
    h = np.zeros((4, 2), np.float16)
    e = np.ones((5, 2), np.float16)
    off = np.array([0, 0, 2, 4, 5], np.int32)
    ids = np.array([1, 5, 2, -1, 3], np.int32)
    got, sc, ws = _csr_call(mf, h, to_dev(e), off, ids)
    assert got.tolist() == [INVALID, INVALID, INVALID, 3]
    assert np.isnan(sc[:3]).all() and sc[3] == 0.0
    assert int(ws.sum()) == 0


def test_rejects_invalid_metadata(mf):
    """tests/cuda/cuda_tests.cu:1283-1339 (host checks before any launch)."""
    import torch

    E = mf.ErrorCode
    rows, hs, v, mx = 1, 4, 8, 2
    hidden = torch.zeros(rows * hs, dtype=torch.float16, device="cuda")
    emb = torch.zeros(v * hs, dtype=torch.float16, device="cuda")
    allowed = torch.zeros(rows * mx, dtype=torch.int32, device="cuda")
    counts = torch.zeros(rows, dtype=torch.int32, device="cuda")
    out = torch.zeros(rows, dtype=torch.int32, device="cuda")
    s = _stream()
    f = mf.restricted_output_head_f16
    assert f(hidden, emb, allowed, counts, out, 0, hs, v, mx, s).code == E.invalid_argument
    assert f(hidden, emb, allowed, counts, out, rows, hs, v, 0, s).code == E.invalid_argument
    assert f(hidden, emb, allowed, counts, out, rows, hs, v, mx, None).code == E.invalid_argument
    assert f(hidden, emb, allowed, counts, counts, rows, hs, v, mx, s).code == E.invalid_argument
    assert f(hidden, emb, allowed, counts, out, 2**64 - 1, hs, v, mx, s).code == E.resource_limit
    assert f(hidden, emb, allowed, counts, out, rows, hs, v, mx, s).ok()


def test_greedy_select_kat(mf, golden_dir):
    """tests/cuda/cuda_tests.cu:508-565 at V = 17 and V = 49,152."""
    import torch
    import sys

    sys.path.insert(0, golden_dir)
    from make_golden import greedy_case

    k = json.load(open(os.path.join(golden_dir, "kat_greedy.json")))
    for case in k["cases"]:
        logits, exp = greedy_case(case["rows"], case["vocabulary_size"])
        assert exp == case["expected"]
        out = torch.empty(case["rows"], dtype=torch.int32, device="cuda")
        st = mf.greedy_select_f16(to_dev(logits), out, case["rows"], case["vocabulary_size"], _stream())
        assert st.ok()
        assert _u32(out).tolist() == exp


def test_greedy_select_rejects(mf):
    """tests/cuda/cuda_tests.cu:1137-1171."""
    import torch

    E = mf.ErrorCode
    logits = torch.zeros(8, dtype=torch.float16, device="cuda")
    tokens = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = _stream()
    assert mf.greedy_select_f16(logits, tokens, 0, 8, s).code == E.invalid_argument
    assert mf.greedy_select_f16(logits, tokens, 1, 8, None).code == E.invalid_argument
    assert mf.greedy_select_f16(logits, tokens, 1, 7, s).code == E.invalid_argument
    assert mf.greedy_select_f16(logits, tokens, 1, 2**32, s).code == E.resource_limit


def test_pr4_logits_greedy(mf, O, golden_dir):
    """Real SmolLM2 logits (tests/fixtures/golden/smollm2-pr4-greedy-f32):
    expected tokens [198, 198, 504]; margins >= 1.0 survive fp16 rounding."""
    import torch

    z = np.load(os.path.join(golden_dir, "pr4_logits.npz"))
    lg = z["logits"].astype(np.float16)
    out = torch.empty(3, dtype=torch.int32, device="cuda")
    assert mf.greedy_select_f16(to_dev(lg), out, 3, lg.shape[1], _stream()).ok()
    assert _u32(out).tolist() == z["tokens"].tolist() == O.greedy_select_f16(lg).tolist()


def test_restricted_greedy_market_dfa(mf, O, golden_dir):
    """tests/cuda/cuda_tests.cu:567-697: real market-DFA states; the
    disallowed logit 100 must lose, an all-NaN row falls back to its lowest id."""
    import torch
    import sys

    sys.path.insert(0, golden_dir)
    from make_golden import market_dfa_case

    z = np.load(os.path.join(golden_dir, "market_dfa.npz"))
    logits, allowed, counts, expected = market_dfa_case(z["state_offsets"], z["arc_tokens"])
    assert np.array_equal(expected, z["select_expected"])
    rows, mx = allowed.shape
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    st = mf.restricted_greedy_select_f16(to_dev(logits), to_dev(allowed), to_dev(counts), out, rows,
                                         logits.shape[1], mx, _stream())
    assert st.ok()
    got = _u32(out)
    assert np.array_equal(got, expected)
    assert np.array_equal(got, O.restricted_greedy_select_f16(logits, allowed, counts, mx))


def test_restricted_greedy_invalid_rows(mf):
    """tests/cuda/cuda_tests.cu:1173-1277."""
    import torch

    E = mf.ErrorCode
    logits = torch.zeros(8, dtype=torch.float16, device="cuda")
    allowed = to_dev(np.array([1, 3, 5, 7], np.uint32))
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    s = _stream()
    for counts, al in (([0], [1, 3, 5, 7]), ([5], [1, 3, 5, 7]), ([2], [1, 8, 5, 7])):
        st = mf.restricted_greedy_select_f16(logits, to_dev(np.array(al, np.uint32)),
                                             to_dev(np.array(counts, np.uint32)), out, 1, 8, 4, s)
        assert st.ok()
        assert _u32(out)[0] == INVALID
    counts = to_dev(np.array([2], np.uint32))
    f = mf.restricted_greedy_select_f16
    assert f(logits, allowed, counts, out, 1, 8, 0, s).code == E.invalid_argument
    assert f(logits, allowed, counts, out, 1, 8, 3, s).code == E.invalid_argument
    assert f(logits, allowed, counts, counts, 1, 8, 4, s).code == E.invalid_argument


# ---- seeded parity against the CPU oracle ---------------------------------

def _ragged_case(seed, rows, kmax, sort_ids=False):
    from market_sim_b200 import synth

    h = synth.hidden_states(seed, rows)
    off, ids = synth.ragged_batch(seed, rows=rows, kmax=kmax, sort_ids=sort_ids)
    return h, off, ids


@pytest.mark.parametrize("rows,kmax,sort_ids", [(1, 1, False), (1, 16, False), (7, 64, True),
                                                (32, 4096, False), (256, 4096, False),
                                                (256, 4096, True)])
def test_csr_parity_vs_oracle(mf, O, emb_full, rows, kmax, sort_ids):
    e, e_dev = emb_full
    h, off, ids = _ragged_case(1000 + rows + kmax, rows, kmax, sort_ids)
    got, sc, ws = _csr_call(mf, h, e_dev, off, ids)
    oid, obest, oru = O.restricted_head_csr(h, e, off, ids, threads=8)
    check_head_parity(got, sc, oid, obest, oru)
    assert int(ws.sum()) == 0


def test_csr_long_single_row_full_vocab(mf, O, emb_full):
    """One row allowing every token (K = 49,152): split over the whole GPU."""
    from market_sim_b200 import synth

    e, e_dev = emb_full
    h = synth.hidden_states(5, 1)
    ids = synth.sample_without_replacement(5, 9, 49_152, 49_152)
    off = np.array([0, ids.size], np.int32)
    got, sc, _ = _csr_call(mf, h, e_dev, off, ids)
    oid, obest, oru = O.restricted_head_csr(h, e, off, ids)
    check_head_parity(got, sc, oid, obest, oru)
    dense, dbest, _ = O.dense_head(h, e)
    assert oid[0] == dense[0]


def test_csr_ties_nan_and_mixed(mf, O):
    """Duplicate embedding rows tie (lowest id wins), NaN hidden rows fall back
    to the lowest candidate, a NaN embedding row never wins, -0 ties +0."""
    from market_sim_b200 import synth

    v = 4096
    e = synth.embedding(77, vocab=v)
    e[100] = e[3000]
    e[200] = np.float16(np.nan)
    e[300] = 0
    e[301] = -0.0
    h = synth.hidden_states(78, 5)
    h[1] = np.float16(np.nan)
    off = np.array([0, 2, 5, 7, 9, 11], np.int32)
    # row 0: exact tie 3000 vs 100 (pick 100); row 1: NaN hidden -> lowest (7)
    # row 2: NaN embedding row 200 with a finite one; row 3: +0 vs -0 rows
    # (scores +0 and -0 tie -> 300); row 4: a plain pair
    ids = np.array([3000, 100, 50, 7, 9000 % v, 200, 5, 301, 300, 11, 12], np.int32)
    got, sc, _ = _csr_call(mf, h, to_dev(e), off, ids)
    oid, obest, oru = O.restricted_head_csr(h, e, off, ids)
    assert got[0] == 100 and oid[0] == 100
    assert got[1] == 7 and oid[1] == 7
    assert got[2] == 5 and oid[2] == 5
    assert got[3] == 300 and oid[3] == 300
    assert got[4] == oid[4]


@pytest.mark.parametrize("rows,kmax", [(16, 256), (3, 16)])
def test_csr_malformed_offsets_gives_sentinel_and_recovers(mf, O, emb_full, rows, kmax):
    """(16, 256): a grid of several blocks, rows decoded by the finishing
    kernel; (3, 16): a one-block grid that finalises its rows itself."""
    import torch

    e, e_dev = emb_full
    h, off, ids = _ragged_case(4, rows, kmax)
    bad = off.copy()
    bad[1] = bad[2] + 1  # decreasing step
    ws = torch.zeros(mf.head_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    got, sc, ws = _csr_call(mf, h, e_dev, bad, ids, ws=ws)
    assert (got == INVALID).all() and np.isnan(sc).all()
    assert int(ws.sum()) == 0
    bad2 = off.copy()
    bad2[-1] -= 1  # last offset does not match the ids size
    got, _, ws = _csr_call(mf, h, e_dev, bad2, ids, ws=ws)
    assert (got == INVALID).all() and int(ws.sum()) == 0
    got, sc, ws = _csr_call(mf, h, e_dev, off, ids, ws=ws)
    oid, obest, oru = O.restricted_head_csr(h, e, off, ids)
    check_head_parity(got, sc, oid, obest, oru)


def test_csr_large_batch_counter_path(mf, O, emb_full):
    """Batches above 4,096 rows take the other merge path (per-row arrival
    counters, in-kernel finaliser, a grid-wide offsets check by the last block
    out): parity with the oracle, an empty row, malformed offsets giving every
    row the sentinel with the workspace left zero, and a good call after it."""
    e, e_dev = emb_full
    rows = 5000
    h, off, ids = _ragged_case(21, rows, 8)
    off = off.copy()
    n7 = off[8] - off[7]  # row 7 empty
    keep = np.ones(ids.size, bool)
    keep[off[7]:off[8]] = False
    ids = ids[keep]
    off[8:] -= n7
    got, sc, ws = _csr_call(mf, h, e_dev, off, ids)
    oid, obest, oru = O.restricted_head_csr(h, e, off, ids)
    check_head_parity(got, sc, oid, obest, oru)
    assert got[7] == INVALID
    assert int(ws.sum()) == 0
    bad = off.copy()
    bad[100] = bad[101] + 1  # decreasing step
    got, sc, ws = _csr_call(mf, h, e_dev, bad, ids, ws=ws)
    assert (got == INVALID).all() and np.isnan(sc).all()
    assert int(ws.sum()) == 0
    got, sc, ws = _csr_call(mf, h, e_dev, off, ids, ws=ws)
    check_head_parity(got, sc, oid, obest, oru)


def test_csr_deterministic_repeats(mf, emb_full):
    _, e_dev = emb_full
    h, off, ids = _ragged_case(9, 128, 4096)
    first = _csr_call(mf, h, e_dev, off, ids)
    for _ in range(5):
        again = _csr_call(mf, h, e_dev, off, ids)
        assert np.array_equal(first[0], again[0])
        assert np.array_equal(first[1].view(np.uint32), again[1].view(np.uint32))


@pytest.mark.parametrize("rows", [1, 16, 256])
@pytest.mark.parametrize("k", [2, 8, 32, 128])
def test_padded_reference_bench_cells(mf, O, emb_full, rows, k):
    """The reference bench's 12 cells (src/tools/cuda_restricted_output_head_bench.cu:129-140):
    patterned hidden rows and ids (row*131 + c*977 + 17) % V, padded table."""
    import torch

    e, e_dev = emb_full
    v = e.shape[0]
    h = np.array([0.5 + (i % 13) / 32.0 for i in range(rows * 576)], np.float32).astype(np.float16)
    allowed = np.array([[(r * 131 + c * 977 + 17) % v for c in range(k)] for r in range(rows)], np.uint32)
    counts = np.full(rows, k, np.uint32)
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    st = mf.restricted_output_head_f16(to_dev(h), e_dev, to_dev(allowed), to_dev(counts), out, rows,
                                       576, v, k, _stream())
    assert st.ok()
    oid, obest = O.restricted_head_padded(h.reshape(rows, 576), e, allowed, counts, k)
    off = np.arange(rows + 1, dtype=np.int32) * k
    _, _, oru = O.restricted_head_csr(h.reshape(rows, 576), e, off, allowed.astype(np.int32).reshape(-1))
    check_head_parity(_u32(out), None, oid, obest, oru)


def test_padded_matches_csr(mf, emb_full):
    """The padded (reference-signature) path and the ragged path agree."""
    import torch

    e, e_dev = emb_full
    h, off, ids = _ragged_case(31, 64, 300)
    rows = 64
    counts = np.diff(off).astype(np.uint32)
    mx = int(counts.max())
    allowed = np.zeros((rows, mx), np.uint32)
    for r in range(rows):
        allowed[r, :counts[r]] = ids[off[r]:off[r + 1]]
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    assert mf.restricted_output_head_f16(to_dev(h), e_dev, to_dev(allowed), to_dev(counts), out, rows,
                                         576, e.shape[0], mx, _stream()).ok()
    got, _, _ = _csr_call(mf, h, e_dev, off, ids)
    assert np.array_equal(_u32(out), got)


@pytest.mark.parametrize("rows,kmax,pad", [(64, 4096, 4096), (3, 2000, 1500), (1, 49_152, 49_152)])
def test_padded_long_tables_match_csr(mf, emb_full, rows, kmax, pad):
    """Tables of more than 512 ids per row go to a cluster of CTAs per row
    (keys merged through distributed shared memory): the same ids as the
    ragged head, and rows whose count is 0 or above the table width give the
    sentinel."""
    import torch

    e, e_dev = emb_full
    if kmax >= 49_152:
        from market_sim_b200 import synth

        h = synth.hidden_states(41, rows)
        off = np.array([0, 49_152], np.int32)
        ids = np.arange(49_152, dtype=np.int32)
    else:
        h, off, ids = _ragged_case(41 + rows, rows, kmax)
    counts = np.diff(off).astype(np.uint32)
    width = max(pad, int(counts.max()))
    allowed = np.zeros((rows, width), np.uint32)
    for r in range(rows):
        allowed[r, :counts[r]] = ids[off[r]:off[r + 1]]
    bad_counts = counts.copy()
    if rows > 2:
        bad_counts[0] = 0
        bad_counts[1] = width + 1
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    assert mf.restricted_output_head_f16(to_dev(h), e_dev, to_dev(allowed), to_dev(bad_counts),
                                         out, rows, 576, e.shape[0], width, _stream()).ok()
    got = _u32(out)
    want, _, _ = _csr_call(mf, h, e_dev, off, ids)
    if rows > 2:
        assert got[0] == INVALID and got[1] == INVALID
        assert np.array_equal(got[2:], want[2:])
    else:
        assert np.array_equal(got, want)


def test_host_pipeline_matches_direct_calls(mf, emb_full):
    """head.HostPipeline (pinned host in/out, overlapped copies) returns the
    same ids and scores as direct device calls, batch after batch."""
    import torch

    e, e_dev = emb_full
    pipe = mf.HostPipeline(e_dev, 256, 600_000, depth=2)
    outs = []
    cases = [_ragged_case(500 + i, 256, 4096) for i in range(5)]
    for h, off, ids in cases:
        oi = torch.empty(256, dtype=torch.int32).pin_memory()
        osc = torch.empty(256, dtype=torch.float32).pin_memory()
        pipe.submit(torch.from_numpy(h).pin_memory(), torch.from_numpy(off).pin_memory(),
                    torch.from_numpy(ids).pin_memory(), oi, osc)
        outs.append((oi, osc))
    pipe.synchronize()
    for (h, off, ids), (oi, osc) in zip(cases, outs):
        got, sc, _ = _csr_call(mf, h, e_dev, off, ids)
        assert np.array_equal(oi.numpy().view(np.uint32), got)
        assert np.array_equal(osc.numpy().view(np.uint32), sc.view(np.uint32))


def test_host_pipeline_packed_batches(mf, emb_full):
    """submit_packed (one H2D and one D2H copy per batch, varying row counts
    and id totals, slots reused) equals direct device calls; a batch whose
    byte count disagrees with its rows and ids is rejected."""
    import torch

    e, e_dev = emb_full
    pipe = mf.HostPipeline(e_dev, 256, 600_000, depth=3)
    cases = [_ragged_case(700 + i, rows, kmax) for i, (rows, kmax) in
             enumerate([(256, 4096), (1, 1), (100, 300), (256, 4096), (7, 4096)])]
    outs = []
    for h, off, ids in cases:
        b = mf.HostPipeline.pack(h, off, ids)
        o = torch.empty(2 * len(h), dtype=torch.int32).pin_memory()
        pipe.submit_packed(b, len(h), ids.size, o)
        outs.append((b, o))
    with pytest.raises(RuntimeError, match="invalid_argument"):
        pipe.submit_packed_ptrs(outs[0][0].data_ptr(), outs[0][0].numel() - 4, 256,
                                cases[0][2].size, outs[0][1].data_ptr())
    pipe.synchronize()
    for (h, off, ids), (_, o) in zip(cases, outs):
        got, sc, _ = _csr_call(mf, h, e_dev, off, ids)
        r = len(h)
        assert np.array_equal(o.numpy()[:r].view(np.uint32), got)
        assert np.array_equal(o.numpy()[r:].view(np.uint32), sc.view(np.uint32))
    pipe.close()


def test_u16_ids_equal_int32_ids(mf, emb_full):
    """The uint16-id layout (``restricted_output_head_csr_u16ids_f16_ex`` and
    the pipeline's ``submit_packed(..., u16_ids=True)``) gives the int32 path's
    ids and scores bit for bit, including a row whose candidate is outside the
    vocabulary (still a u16 value) and an empty row."""
    import torch

    e, e_dev = emb_full
    vocab = int(e_dev.shape[0])
    pipe = mf.HostPipeline(e_dev, 256, 600_000, depth=2)
    for i, (rows, kmax) in enumerate([(256, 4096), (1, 1), (33, 300)]):
        h, off, ids = _ragged_case(1300 + i, rows, kmax)
        if rows == 33:  # row 5: an id past the vocabulary; row 6: empty
            ids = ids.copy()
            ids[off[5]] = vocab + 7
            keep = np.ones(ids.size, bool)
            keep[off[6]:off[7]] = False
            n6 = off[7] - off[6]
            ids = ids[keep]
            off = off.copy()
            off[7:] -= n6
        want, want_sc, _ = _csr_call(mf, h, e_dev, off, ids)
        out = torch.empty(rows, dtype=torch.int32, device="cuda")
        sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        ws = torch.zeros(mf.head_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
        ids16 = torch.from_numpy(ids.astype(np.uint16).view(np.int16)).cuda()
        st = mf.restricted_output_head_csr_u16ids_f16_ex(to_dev(h), e_dev, to_dev(off), ids16, out,
                                                         sc, ws, rows, 576, vocab, 0, _stream())
        assert st.ok(), st
        torch.cuda.synchronize()
        assert np.array_equal(_u32(out), want)
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), want_sc.view(np.uint32))
        assert int(ws.sum()) == 0  # the workspace is left zero
        b = mf.HostPipeline.pack(h, off, ids, u16_ids=True)
        o = torch.empty(2 * rows, dtype=torch.int32).pin_memory()
        pipe.wait(pipe.submit_packed(b, rows, ids.size, o, u16_ids=True))
        assert np.array_equal(o.numpy()[:rows].view(np.uint32), want)
        assert np.array_equal(o.numpy()[rows:].view(np.uint32), want_sc.view(np.uint32))
    with pytest.raises(RuntimeError, match="invalid_argument"):  # byte count of int32 ids
        b32 = mf.HostPipeline.pack(h, off, ids)
        pipe.submit_packed(b32, 33, ids.size, o, u16_ids=True)
    pipe.close()


def test_u16_ids_generic_width(mf):
    """The uint16-id entry on the generic (any hidden width) kernel equals the
    int32 entry bit for bit: 9 rows of width 40 over a 300-row table."""
    import torch

    rng = np.random.default_rng(5)
    rows, width, vocab = 9, 40, 300
    h = torch.from_numpy(rng.standard_normal((rows, width)).astype(np.float16)).cuda()
    emb = torch.from_numpy((0.1 * rng.standard_normal((vocab, width))).astype(np.float16)).cuda()
    counts = rng.integers(0, 30, rows)
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    ids = rng.integers(0, vocab, int(off[-1])).astype(np.int32)
    outs = []
    for u16 in (False, True):
        out = torch.empty(rows, dtype=torch.int32, device="cuda")
        sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        ws = torch.zeros(mf.head_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
        if u16:
            d = torch.from_numpy(ids.astype(np.uint16).view(np.int16)).cuda()
            st = mf.restricted_output_head_csr_u16ids_f16_ex(h, emb, to_dev(off), d, out, sc, ws,
                                                             rows, width, vocab, 0, _stream())
        else:
            st = mf.restricted_output_head_csr_f16_ex(h, emb, to_dev(off), to_dev(ids), out, sc, ws,
                                                      rows, width, vocab, 0, _stream())
        assert st.ok(), st
        torch.cuda.synchronize()
        outs.append((_u32(out), sc.cpu().numpy().view(np.uint32)))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])
    assert (outs[0][0][counts == 0] == INVALID).all()


def test_host_pipeline_wait_on_reused_slot(mf, emb_full):
    """More batches than slots, then wait(ticket 0) alone: the first batch's
    slot has been reused since, and wait must still not return before that
    batch's results are home (its slot's stream holds them in order)."""
    import torch

    e, e_dev = emb_full
    depth = 2
    pipe = mf.HostPipeline(e_dev, 256, 600_000, depth=depth)
    cases = [_ragged_case(900 + i, 256, 4096) for i in range(2 * depth + 1)]
    outs, tickets = [], []
    for h, off, ids in cases:
        b = mf.HostPipeline.pack(h, off, ids)
        o = torch.full((2 * len(h),), -7, dtype=torch.int32).pin_memory()
        tickets.append(pipe.submit_packed(b, len(h), ids.size, o))
        outs.append((b, o))
    pipe.wait(tickets[0])
    h, off, ids = cases[0]
    got = outs[0][1].numpy()[:256].view(np.uint32).copy()
    pipe.synchronize()
    want, _, _ = _csr_call(mf, h, e_dev, off, ids)
    assert np.array_equal(got, want)
    pipe.close()


@pytest.mark.parametrize("rows,kmax,hs", [(64, 4096, 576), (9, 40, 64)])
def test_fused_rmsnorm_head_vs_oracle(mf, O, rows, kmax, hs):
    """Final RMSNorm fused into the head: equals the oracle's rms_norm_f32
    (src/cpu/operators.cpp:489-537), rounded to fp16 as rms_norm_f16 stores
    it, followed by the restricted head (margin rule for near-ties)."""
    import torch

    from market_sim_b200 import synth

    vocab = 49_152 if hs == 576 else 3000
    e = synth.embedding(61 + hs, vocab=vocab, hidden=hs)
    x = (synth.normal(62, 1, rows * hs) * 3).astype(np.float32).astype(np.float16).reshape(rows, hs)
    g = synth.normal(63, 2, hs, 1.0, 0.02).astype(np.float32).astype(np.float16)
    off, ids = synth.ragged_batch(64, rows=rows, kmax=kmax, vocab=vocab)
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    ws = torch.zeros(mf.head_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    st = mf.restricted_output_head_csr_rmsnorm_f16(to_dev(x), to_dev(g), 1e-5, to_dev(e),
                                                   to_dev(off), to_dev(ids), out, sc, ws, rows, hs,
                                                   vocab, _stream())
    assert st.ok(), st
    torch.cuda.synchronize()
    h16 = O.rms_norm_f32(O.widen(x), O.widen(g), 1e-5).astype(np.float16)
    oid, obest, oru = O.restricted_head_csr(h16, e, off, ids)
    check_head_parity(_u32(out), sc.cpu().numpy(), oid, obest, oru)
    assert int(ws.sum()) == 0


def test_fused_rmsnorm_rejects(mf):
    import torch

    E = mf.ErrorCode
    rows, hs, v = 2, 576, 100
    x = torch.zeros((rows, hs), dtype=torch.float16, device="cuda")
    g = torch.ones(hs, dtype=torch.float16, device="cuda")
    e = torch.zeros((v, hs), dtype=torch.float16, device="cuda")
    off = to_dev(np.array([0, 1, 2], np.int32))
    ids = to_dev(np.array([3, 4], np.int32))
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    ws = torch.zeros(mf.head_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    s = _stream()
    f = mf.restricted_output_head_csr_rmsnorm_f16
    assert f(x, g, 0.0, e, off, ids, out, None, ws, rows, hs, v, s).code == E.invalid_argument
    assert f(x, g, float("nan"), e, off, ids, out, None, ws, rows, hs, v, s).code == E.invalid_argument
    assert f(x, g[:100], 1e-5, e, off, ids, out, None, ws, rows, hs, v, s).code == E.invalid_argument
    assert f(x, g, 1e-5, e, off, ids, out, None, ws, rows, hs, v, s).ok()


def test_overlapped_launches_match_plain_calls(mf, emb_full):
    """MF_LAUNCH_OVERLAP_PREVIOUS: back-to-back launches on independent
    batches sharing one workspace (eagerly and inside a CUDA graph), each
    writing its own outputs or all writing the same ones, equal plain calls;
    the workspace is left zero; unknown flag bits are rejected."""
    import torch

    e, e_dev = emb_full
    cases = [_ragged_case(800 + i, rows, kmax) for i, (rows, kmax) in
             enumerate([(256, 4096), (256, 4096), (64, 512), (256, 4096), (3, 40), (256, 2048)])]
    want = [_csr_call(mf, h, e_dev, off, ids)[:2] for h, off, ids in cases]
    dev = [(to_dev(h), to_dev(off), to_dev(ids)) for h, off, ids in cases]
    ws = torch.zeros(mf.head_workspace_bytes(256), dtype=torch.uint8, device="cuda")
    s = gpu_stream()
    flag = mf.LAUNCH_OVERLAP_PREVIOUS

    def launch(j, out, sc):
        h, off, ids = dev[j]
        st = mf.restricted_output_head_csr_f16_ex(h, e_dev, off, ids, out, sc, ws, len(cases[j][0]),
                                                  576, 49_152, flag, s)
        assert st.ok(), st

    outs = [(torch.empty(len(c[0]), dtype=torch.int32, device="cuda"),
             torch.empty(len(c[0]), dtype=torch.float32, device="cuda")) for c in cases]
    with torch.cuda.stream(s):
        for rep in range(4):
            for j in range(len(cases)):
                launch(j, *outs[j])
    s.synchronize()
    for (o, sc), (wi, ws_) in zip(outs, want):
        assert np.array_equal(_u32(o), wi)
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), ws_.view(np.uint32))
    assert int(ws.sum()) == 0

    shared = (torch.empty(256, dtype=torch.int32, device="cuda"),
              torch.empty(256, dtype=torch.float32, device="cuda"))
    g = torch.cuda.CUDAGraph()
    order = [0, 1, 3, 5, 0, 1, 3, 5, 1, 3]  # all 256-row batches; the last one wins
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for j in order:
                launch(j, *shared)
        for _ in range(3):
            g.replay()
    s.synchronize()
    assert np.array_equal(_u32(shared[0]), want[order[-1]][0])
    assert int(ws.sum()) == 0

    h, off, ids = dev[0]
    st = mf.restricted_output_head_csr_f16_ex(h, e_dev, off, ids, *shared, ws, 256, 576, 49_152,
                                              2, s)
    assert st.code == mf.ErrorCode.invalid_argument

    # a malformed batch (decreasing offsets) between good ones: every row of
    # it gets the sentinel, the workspace is cleared, the next batch is exact
    bad_off = cases[0][1].copy()
    assert bad_off[5] > 0
    bad_off[6] = bad_off[5] - 1  # row 5 ends before it starts
    bad = to_dev(bad_off)
    o_bad = (torch.empty(256, dtype=torch.int32, device="cuda"),
             torch.empty(256, dtype=torch.float32, device="cuda"))
    with torch.cuda.stream(s):
        launch(0, *outs[0])
        st = mf.restricted_output_head_csr_f16_ex(h, e_dev, bad, ids, *o_bad, ws, 256, 576,
                                                  49_152, flag, s)
        assert st.ok(), st
        launch(1, *outs[1])
    s.synchronize()
    assert (_u32(o_bad[0]) == INVALID).all()
    assert np.array_equal(_u32(outs[0][0]), want[0][0])
    assert np.array_equal(_u32(outs[1][0]), want[1][0])
    assert int(ws.sum()) == 0


def test_padded_long_table_generic_width(mf):
    """The cluster-split padded head on the generic (non-576) path: a
    64-wide model, 1,500-id tables, equals the ragged head."""
    import torch

    from market_sim_b200 import synth

    v, hs, rows = 3000, 64, 5
    e = synth.embedding(77, vocab=v, hidden=hs)
    e_dev = to_dev(e)
    h = synth.hidden_states(78, rows, hs)
    off, ids = synth.ragged_batch(79, rows=rows, kmax=1500, vocab=v)
    counts = np.diff(off).astype(np.uint32)
    allowed = np.zeros((rows, 1500), np.uint32)
    for r in range(rows):
        allowed[r, :counts[r]] = ids[off[r]:off[r + 1]]
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    assert mf.restricted_output_head_f16(to_dev(h), e_dev, to_dev(allowed), to_dev(counts), out,
                                         rows, hs, v, 1500, _stream()).ok()
    want, _, _ = _csr_call(mf, h, e_dev, off, ids)
    assert np.array_equal(_u32(out), want)
