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


class _Exchange:
    """Exchange buffers given as raw pointers (both on this GPU)."""

    def __init__(self, ptrs, nbytes, world, rank):
        self.ptrs, self.nbytes, self.world, self.rank = ptrs, nbytes, world, rank


def _slot(buf, rows, world, epoch, q):
    """Rank q's keys for call `epoch` inside one exchange buffer (u64 view)."""
    par = epoch & 1
    off = 512 + (par * world + q) * rows * 8
    return buf[off:off + rows * 8].view(dtype=__import__("torch").int64)


def _flag(buf, q):
    """Rank q's flag in one exchange buffer: 2 x epoch + failed."""
    import torch

    return buf[64 + 4 * q:64 + 4 * q + 4].view(torch.int32)


def _broken(buf):
    return int(buf[4:8].view(__import__("torch").int32).item())


def test_dense_sharded_merge_emulated_peer(mf):
    """In-kernel vocabulary-shard merge on one GPU: rank 1's keys and flag
    are stored into rank 0's exchange buffer beforehand (as rank 1 would over
    NVLink), so rank 0's kernel never waits on another launch.  Over three
    calls (epochs 1-3, both slot parities) rank 0's ids / scores / keys equal
    the unsharded head, and rank 0's keys and flag (2 x epoch) land in the
    peer buffer."""
    import torch

    from market_sim_b200 import synth

    rows, vocab, hs, world = 256, 8192, 576, 2
    per = vocab // world
    e = synth.embedding(91, vocab=vocab)
    h = synth.hidden_states(92, rows)
    e_d, h_d = to_dev(e), to_dev(h)
    full_keys, full_ids, full_sc = _dense(mf, h_d, e_d, rows, hs, vocab)
    k0, _, _ = _dense(mf, h_d, e_d[:per].contiguous(), rows, hs, per, 0)
    k1, _, _ = _dense(mf, h_d, e_d[per:].contiguous(), rows, hs, per, per)
    nbytes = mf.exchange_bytes(rows, world)
    own = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    peer = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    ex = _Exchange([own.data_ptr(), peer.data_ptr()], nbytes, world, 0)
    shard0 = e_d[:per].contiguous()
    ws = torch.zeros(mf.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    for epoch in (1, 2, 3):
        _slot(own, rows, world, epoch, 1).copy_(torch.from_numpy(k1.view(np.int64)))
        _flag(own, 1).fill_(2 * epoch)
        keys = torch.empty(rows, dtype=torch.int64, device="cuda")
        ids = torch.empty(rows, dtype=torch.int32, device="cuda")
        sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        st = mf.dense_head_sharded_f16(h_d, shard0, keys, ids, sc, ws, rows, hs, per, 0, ex,
                                       gpu_stream())
        assert st.ok(), st
        torch.cuda.synchronize()
        assert np.array_equal(keys.cpu().numpy().view(np.uint64), full_keys)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), full_ids)
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), full_sc.view(np.uint32))
        assert np.array_equal(_slot(peer, rows, world, epoch, 0).cpu().numpy().view(np.uint64), k0)
        assert int(_flag(peer, 0).item()) == 2 * epoch
        assert int(own[:4].view(torch.int32).item()) == epoch
        assert _broken(own) == 0
        assert int(ws.sum()) == 0


def test_dense_sharded_peer_never_arrives(mf):
    """A peer that never stores its keys: the wait runs out after 100 ms, the
    rows get the sentinel on this rank, and the context stays usable."""
    import torch

    from market_sim_b200 import synth

    rows, vocab, hs, world = 128, 1024, 576, 2
    e_d = to_dev(synth.embedding(93, vocab=vocab))
    h_d = to_dev(synth.hidden_states(94, rows))
    nbytes = mf.exchange_bytes(rows, world)
    own = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    peer = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    ex = _Exchange([own.data_ptr(), peer.data_ptr()], nbytes, world, 0)
    ids = torch.zeros(rows, dtype=torch.int32, device="cuda")
    ws = torch.zeros(mf.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    st = mf.dense_head_sharded_f16(h_d, e_d, None, ids, None, ws, rows, hs, vocab, 0, ex,
                                   gpu_stream())
    assert st.ok(), st
    torch.cuda.synchronize()
    assert (ids.cpu().numpy().view(np.uint32) == INVALID).all()
    assert int(ws.sum()) == 0
    assert _broken(own) == 1 and mf.exchange_broken(own) == 1
    _, ids2, _ = _dense(mf, h_d, e_d, rows, hs, vocab)
    assert (ids2 < vocab).all()


def test_dense_sharded_stale_or_failed_peer_gives_sentinel(mf):
    """Exact epoch match: a peer flag naming another call (two calls ahead)
    never passes, so the wait runs out and every row gets the sentinel
    instead of decoding keys of another call; a peer flag with the failed
    bit set gives the sentinel at once.  Either way the buffer is marked
    broken and later calls on it give the sentinel too."""
    import torch

    from market_sim_b200 import synth

    rows, vocab, hs, world = 128, 1024, 576, 2
    e_d = to_dev(synth.embedding(97, vocab=vocab))
    h_d = to_dev(synth.hidden_states(98, rows))
    nbytes = mf.exchange_bytes(rows, world)
    ws = torch.zeros(mf.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    for flag in (2 * 3, 2 * 1 + 1):  # epoch 3 while this call is epoch 1; epoch 1 failed
        own = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        peer = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        ex = _Exchange([own.data_ptr(), peer.data_ptr()], nbytes, world, 0)
        _flag(own, 1).fill_(flag)
        ids = torch.zeros(rows, dtype=torch.int32, device="cuda")
        st = mf.dense_head_sharded_f16(h_d, e_d, None, ids, None, ws, rows, hs, vocab, 0, ex,
                                       gpu_stream())
        assert st.ok(), st
        torch.cuda.synchronize()
        assert (ids.cpu().numpy().view(np.uint32) == INVALID).all()
        assert _broken(own) == 1
        _flag(own, 1).fill_(2 * 2)  # even a matching flag for the next call: still broken
        st = mf.dense_head_sharded_f16(h_d, e_d, None, ids, None, ws, rows, hs, vocab, 0, ex,
                                       gpu_stream())
        assert st.ok(), st
        torch.cuda.synchronize()
        assert (ids.cpu().numpy().view(np.uint32) == INVALID).all()
        assert int(ws.sum()) == 0


def test_dense_sharded_rejects(mf):
    import torch

    E = mf.ErrorCode
    rows, hs, vocab = 128, 64, 256
    h = torch.zeros((rows, hs), dtype=torch.float16, device="cuda")
    e = torch.zeros((vocab, hs), dtype=torch.float16, device="cuda")
    ids = torch.zeros(rows, dtype=torch.int32, device="cuda")
    ws = torch.zeros(mf.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    nb = mf.exchange_bytes(rows, 2)
    a = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    b = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    s = gpu_stream()
    call = lambda ex: mf.dense_head_sharded_f16(h, e, None, ids, None, ws, rows, hs, vocab, 0, ex, s)
    assert call(_Exchange([a.data_ptr(), b.data_ptr()], nb, 2, 2)).code == E.invalid_argument
    assert call(_Exchange([a.data_ptr(), a.data_ptr()], nb, 2, 0)).code == E.invalid_argument
    assert call(_Exchange([a.data_ptr(), b.data_ptr()], nb - 8, 2, 0)).code == E.invalid_argument
    assert call(_Exchange([a.data_ptr(), b.data_ptr() + 8], nb, 2, 0)).code == E.invalid_argument
    assert call(_Exchange([a.data_ptr()] * 9, nb, 9, 0)).code == E.resource_limit


def test_dense_overlapped_launches_match_plain_calls(mf):
    """MF_LAUNCH_OVERLAP_PREVIOUS: back-to-back dense launches on independent
    hidden batches sharing one workspace equal plain calls, eagerly and in a
    CUDA graph; the workspace is left zero; unknown flag bits are rejected."""
    import torch

    from market_sim_b200 import synth

    rows, vocab, hs = 512, 8192, 576
    e_d = to_dev(synth.embedding(95, vocab=vocab))
    hids = [to_dev(synth.hidden_states(96 + j, rows)) for j in range(4)]
    want = [_dense(mf, h, e_d, rows, hs, vocab, want_keys=False)[1] for h in hids]
    ws = torch.zeros(mf.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    outs = [torch.empty(rows, dtype=torch.int32, device="cuda") for _ in hids]
    s = gpu_stream()
    flag = mf.LAUNCH_OVERLAP_PREVIOUS

    def launch(j, out):
        st = mf.dense_head_f16_ex(hids[j], e_d, None, out, None, ws, rows, hs, vocab, 0, flag, s)
        assert st.ok(), st

    with torch.cuda.stream(s):
        for _ in range(3):
            for j in range(len(hids)):
                launch(j, outs[j])
    s.synchronize()
    for o, w in zip(outs, want):
        assert np.array_equal(o.cpu().numpy().view(np.uint32), w)
    assert int(ws.sum()) == 0
    shared = torch.empty(rows, dtype=torch.int32, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for j in (0, 1, 2, 3, 2, 1):
                launch(j, shared)
        g.replay()
        g.replay()
    s.synchronize()
    assert np.array_equal(shared.cpu().numpy().view(np.uint32), want[1])
    assert int(ws.sum()) == 0
    st = mf.dense_head_f16_ex(hids[0], e_d, None, shared, None, ws, rows, hs, vocab, 0, 4, s)
    assert st.code == mf.ErrorCode.invalid_argument
