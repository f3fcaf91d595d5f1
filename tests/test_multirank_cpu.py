"""Host logic of the vocabulary-sharded dense head on CPU: two gloo ranks
each take the oracle argmax over their vocabulary shard, pack (score, id)
keys, merge with a signed MAX all-reduce of the sign-flipped keys — the
collective bench.py issues over NCCL — and must equal the unsharded oracle.
Also checks the key encoding against the selection rule."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.multiprocessing as mp

from market_sim_b200 import keys as K


def test_key_order_is_the_selection_rule():
    s = np.array([1.0, 1.0, -0.0, 0.0, np.nan, -np.inf, np.inf, -2.0], np.float32)
    i = np.array([7, 3, 9, 4, 1, 2, 5, 0], np.uint32)
    k = K.pack(s, i)
    order = np.argsort(-k.astype(np.float64), kind="stable")  # descending key
    assert i[order[0]] == 5                      # +inf wins
    assert k[1] > k[0]                           # tie at 1.0: lower id wins
    assert k[3] > k[2]                           # +0 / -0 tie: lower id (4) wins
    assert (k[4] < k[np.arange(8) != 4]).all()   # NaN below every real score
    ids, sc = K.unpack(k)
    assert np.array_equal(ids, i) and np.array_equal(sc[~np.isnan(s)], np.where(s == 0, 0, s)[~np.isnan(s)])
    signed = K.to_signed(k)
    assert np.array_equal(np.argsort(signed, kind="stable"), np.argsort(k, kind="stable"))
    assert np.array_equal(K.from_signed(signed), k)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist

    from market_sim_b200 import keys as K
    from market_sim_b200 import synth
    from oracle import oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    vocab, rows = 2048, 24
    e = synth.embedding(11, vocab=vocab)
    h = synth.hidden_states(12, rows)
    per = vocab // world
    ids, best, _ = O.dense_head(h, e, rank * per, (rank + 1) * per)
    k = torch.from_numpy(K.to_signed(K.pack(best, ids)).copy())
    dist.all_reduce(k, op=dist.ReduceOp.MAX)
    if rank == 0:
        m_ids, m_sc = K.unpack(K.from_signed(k.numpy()))
        out["ids"] = m_ids.tolist()
    dist.destroy_process_group()


def test_two_gloo_ranks_merge_vocab_shards():
    from market_sim_b200 import synth
    from oracle import oracle as O

    port = _free_port()
    with mp.Manager() as man:
        out = man.dict()
        mp.spawn(_rank, args=(2, port, out), nprocs=2, join=True)
        merged = out["ids"]
    e = synth.embedding(11, vocab=2048)
    h = synth.hidden_states(12, 24)
    full, _, _ = O.dense_head(h, e)
    assert merged == full.tolist()


class _FakeExchangeLib:
    """The real library for everything but the four CUDA calls of the
    exchange setup, which are faked: rank r's buffer is at 0x10000 * (r + 1),
    its 64-byte handle names r, and opening a handle maps it to 0x900000 + r
    (or fails for the rank in `fail_open`)."""

    def __init__(self, real, rank, fail_open=None):
        self._real, self.rank, self.fail_open = real, rank, fail_open
        self.calls = []

    def __getattr__(self, name):
        return getattr(self._real, name)

    def mf_exchange_alloc(self, buf_ref, nbytes, handle):
        import ctypes

        from market_sim_b200._lib import MfStatus

        self.calls.append(("alloc", int(nbytes)))
        ctypes.cast(buf_ref, ctypes.POINTER(ctypes.c_void_p))[0] = 0x10000 * (self.rank + 1)
        ctypes.memmove(handle, bytes([self.rank]) + b"h" * 63, 64)
        return MfStatus(0, 0)

    def mf_exchange_open_peer(self, handle, peer_ref):
        import ctypes

        from market_sim_b200._lib import MfStatus

        q = ctypes.string_at(handle, 64)[0]
        self.calls.append(("open", q))
        if q == self.fail_open:
            return MfStatus(22, 1)
        ctypes.cast(peer_ref, ctypes.POINTER(ctypes.c_void_p))[0] = 0x900000 + q
        return MfStatus(0, 0)

    def mf_exchange_close_peer(self, p):
        self.calls.append(("close", int(p)))

    def mf_exchange_free(self, p):
        self.calls.append(("free", int(p)))


def _exchange_rank(rank, world, port, out):
    import torch.distributed as dist

    from market_sim_b200 import head

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    real = head.lib
    try:
        fake = _FakeExchangeLib(real, rank)
        head.lib = fake
        ex = head.VocabShardExchange(100)
        out[f"ptrs{rank}"] = list(ex.ptrs)
        out[f"nbytes{rank}"] = ex.nbytes
        ex.close()
        out[f"calls{rank}"] = list(fake.calls)
        # a peer whose buffer cannot be mapped: the constructor raises and
        # releases what it had opened and its own buffer
        fake = _FakeExchangeLib(real, rank, fail_open=world - 1 if rank != world - 1 else None)
        head.lib = fake
        try:
            head.VocabShardExchange(100)
            out[f"raised{rank}"] = False
        except RuntimeError:
            out[f"raised{rank}"] = True
        out[f"calls_fail{rank}"] = list(fake.calls)
    finally:
        head.lib = real
        dist.destroy_process_group()


def test_vocab_shard_exchange_setup_three_gloo_ranks():
    """head.VocabShardExchange on three gloo ranks with the CUDA calls faked:
    the IPC handles are all-gathered, every rank maps every peer's buffer and
    keeps its own at its rank's position, close() unmaps and frees, and a
    failed mapping raises after releasing everything."""
    from market_sim_b200 import head

    world = 3
    port = _free_port()
    with mp.Manager() as man:
        out = man.dict()
        mp.spawn(_exchange_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        want = [0x10000 * (r + 1) if q == r else 0x900000 + q for q in range(world)]
        assert res[f"ptrs{r}"] == want
        assert res[f"nbytes{r}"] == head.exchange_bytes(100, world) == 512 + 2 * world * 100 * 8
        calls = res[f"calls{r}"]
        assert calls[0] == ("alloc", res[f"nbytes{r}"])
        assert sorted(c for c in calls if c[0] == "open") == [("open", q) for q in range(world)
                                                               if q != r]
        assert ("free", 0x10000 * (r + 1)) in calls
        assert sum(c[0] == "close" for c in calls) == world - 1
        failing = r != world - 1
        assert res[f"raised{r}"] == failing
        if failing:
            cf = res[f"calls_fail{r}"]
            opened = [c for c in cf if c[0] == "open" and c[1] != world - 1]
            assert sum(c[0] == "close" for c in cf) == len(opened)
            assert ("free", 0x10000 * (r + 1)) in cf
