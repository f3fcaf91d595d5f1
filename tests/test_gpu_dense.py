"""GPU parity of the dense full-vocabulary head (tcgen05 GEMM + fused argmax)
through the C-ABI: against the FP32 CPU oracle (full logits, argmax) at
sizes the oracle finishes in seconds, against a torch FP32 matmul at the
benchmark size (B = 1024, V = 49,152), and the vocabulary-shard merge
(max of packed keys) against the unsharded result."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import INVALID, check_head_parity, gpu_stream, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf(cuda):
    from market_sim_b200 import head

    return head


def _dense(mf, hid_d, emb_d, rows, hs, vrows, vbegin=0, want_keys=True):
    import torch

    keys = torch.empty(rows, dtype=torch.int64, device="cuda") if want_keys else None
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    ws = torch.zeros(mf.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    st = mf.dense_head_f16(hid_d, emb_d, keys, ids, sc, ws, rows, hs, vrows, vbegin, gpu_stream())
    assert st.ok(), st
    torch.cuda.synchronize()
    assert int(ws.sum()) == 0, "workspace must be left zero"
    return (None if keys is None else keys.cpu().numpy().view(np.uint64),
            ids.cpu().numpy().view(np.uint32), sc.cpu().numpy())


@pytest.mark.parametrize("rows,vocab,hs", [(128, 256, 576), (200, 1000, 576), (256, 4096, 576),
                                           (37, 777, 64), (130, 513, 320)])
def test_dense_vs_oracle(mf, rows, vocab, hs):
    from market_sim_b200 import synth
    from oracle import oracle as O

    e = synth.embedding(rows + vocab, vocab=vocab, hidden=hs)
    h = synth.hidden_states(rows * 3 + hs, rows, hidden=hs)
    _, ids, sc = _dense(mf, to_dev(h), to_dev(e), rows, hs, vocab)
    oid, obest, oru = O.dense_head(h, e)
    check_head_parity(ids, sc, oid, obest, oru)


def test_dense_ties_nan_rows(mf):
    """Duplicate embedding rows tie (lowest id wins), an all-NaN hidden row
    selects the first id, a NaN embedding row never wins."""
    from market_sim_b200 import synth
    from oracle import oracle as O

    rows, vocab, hs = 128, 600, 576
    e = synth.embedding(5, vocab=vocab, hidden=hs)
    h = synth.hidden_states(6, rows, hidden=hs)
    e[300] = np.float16(np.nan)
    e[450] = e[17]
    h[3] = np.float16(np.nan)
    h[4] = (e[17].astype(np.float32) * 40).astype(np.float16)  # 17 and 450 tie at the top
    _, ids, sc = _dense(mf, to_dev(h), to_dev(e), rows, hs, vocab)
    oid, obest, oru = O.dense_head(h, e)
    assert ids[3] == 0 and oid[3] == 0 and np.isnan(sc[3])
    assert ids[4] == 17 and oid[4] == 17
    assert (ids != 300).all()
    check_head_parity(ids, sc, oid, obest, oru)


def test_dense_full_size_vs_torch(mf):
    """B = 1024 x V = 49,152 x 576: ids equal a torch FP32 reference argmax
    except within the 1e-3 margin; scores within 2e-3 relative."""
    import torch

    from market_sim_b200 import synth

    rows, vocab, hs = 1024, 49_152, 576
    e = synth.embedding(2025)
    h = synth.hidden_states(2026, rows)
    e_d, h_d = to_dev(e), to_dev(h)
    _, ids, sc = _dense(mf, h_d, e_d, rows, hs, vocab)
    logits = h_d.float() @ e_d.float().T
    top2 = torch.topk(logits, 2, dim=1)
    ref_ids = torch.argmax(logits, dim=1).cpu().numpy().astype(np.uint32)
    best = top2.values[:, 0].cpu().numpy()
    ru = top2.values[:, 1].cpu().numpy()
    check_head_parity(ids, sc, ref_ids, best, ru)


def test_dense_vocab_shards_merge(mf):
    """Four vocabulary shards (each its own call with vocab_begin) merged by
    a signed max of the sign-flipped keys equal the unsharded head."""
    import torch

    from market_sim_b200 import synth

    rows, vocab, hs, shards = 256, 8192, 576, 4
    e = synth.embedding(77, vocab=vocab)
    h = synth.hidden_states(78, rows)
    e_d, h_d = to_dev(e), to_dev(h)
    full_keys, full_ids, full_sc = _dense(mf, h_d, e_d, rows, hs, vocab)
    per = vocab // shards
    merged = torch.full((rows,), -(2**63), dtype=torch.int64, device="cuda")
    for s in range(shards):
        k, ids_s, _ = _dense(mf, h_d, e_d[s * per:(s + 1) * per].contiguous(), rows, hs, per, s * per)
        assert ((ids_s >= s * per) & (ids_s < (s + 1) * per)).all()
        kt = torch.from_numpy(k.view(np.int64).copy()).cuda() ^ mf.KEY_SIGN_FLIP - 2**64
        merged = torch.maximum(merged, kt)
    merged = (merged ^ (mf.KEY_SIGN_FLIP - 2**64)).contiguous()
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    assert mf.decode_keys(merged, out, sc, rows, gpu_stream()).ok()
    torch.cuda.synchronize()
    assert np.array_equal(merged.cpu().numpy().view(np.uint64), full_keys)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), full_ids)


def test_dense_rejects(mf):
    import torch

    E = mf.ErrorCode
    h = torch.zeros((4, 100), dtype=torch.float16, device="cuda")
    e = torch.zeros((8, 100), dtype=torch.float16, device="cuda")
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws = torch.zeros(mf.dense_workspace_bytes(4), dtype=torch.uint8, device="cuda")
    s = gpu_stream()
    assert mf.dense_head_f16(h, e, None, ids, None, ws, 4, 100, 8, 0, s).code == E.resource_limit
    assert mf.dense_head_f16(h, e, None, ids, None, ws, 0, 100, 8, 0, s).code == E.invalid_argument
    h64 = torch.zeros((4, 64), dtype=torch.float16, device="cuda")
    e64 = torch.zeros((8, 64), dtype=torch.float16, device="cuda")
    assert mf.dense_head_f16(h64, e64, None, None, None, ws, 4, 64, 8, 0, s).code == E.invalid_argument
    assert mf.dense_head_f16(h64, e64, None, ids, None, ws, 4, 64, 8, 0, None).code == E.invalid_argument
    assert mf.dense_head_f16(h64, e64, None, ids, None, ws, 4, 64, 8, 0, s).ok()
    assert INVALID == 0xFFFFFFFF


def test_dense_bounded_waits_give_up_cleanly(mf):
    """Failure detection without a GPU fault: the kernel's producer issues no
    loads (a barrier that nothing completes), its waits run out after 100 ms,
    every row gets the sentinel, the error word is reported, and the context
    stays usable for the next call."""
    import ctypes

    import torch

    from market_sim_b200._lib import lib

    err, bad = ctypes.c_uint32(7), ctypes.c_uint32(0)
    s = gpu_stream()
    st = lib.mf_dense_selftest_wait_timeout(ctypes.c_void_p(s.cuda_stream), ctypes.byref(err),
                                            ctypes.byref(bad))
    assert st.code == 0, (st.code, st.detail)
    assert err.value == 1 and bad.value == 128
    # the context is still healthy: a normal dense call succeeds
    from market_sim_b200 import synth

    e = synth.embedding(3, vocab=300)
    h = synth.hidden_states(4, 64)
    _, ids, _ = _dense(mf, to_dev(h), to_dev(e), 64, 576, 300)
    assert (ids < 300).all()
    torch.cuda.synchronize()
