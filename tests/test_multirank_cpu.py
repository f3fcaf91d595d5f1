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
