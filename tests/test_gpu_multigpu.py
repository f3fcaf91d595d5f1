"""Vocabulary-sharded dense head on two GPUs, one process per GPU: the
in-kernel merge over NVLink (CUDA IPC exchange buffers) equals the
unsharded head computed locally, call after call; and it equals the NCCL
max all-reduce of the keys.  Skipped unless two GPUs are visible."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        from market_sim_b200 import head, synth

        rows, vocab, hs = 512, 49_152, 576
        per = vocab // world
        e = torch.from_numpy(synth.embedding(2027)).cuda()
        shard = e[rank * per:(rank + 1) * per].contiguous()
        ex = head.VocabShardExchange(rows)
        s = torch.cuda.Stream()
        ws = torch.zeros(head.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
        ok = True
        for call in range(6):
            h = torch.from_numpy(synth.hidden_states(3000 + call, rows)).cuda()
            keys = torch.empty(rows, dtype=torch.int64, device="cuda")
            ids = torch.empty(rows, dtype=torch.int32, device="cuda")
            st = head.dense_head_sharded_f16(h, shard, keys, ids, None, ws, rows, hs, per,
                                             rank * per, ex, s.cuda_stream)
            assert st.ok(), st
            ref_k = torch.empty(rows, dtype=torch.int64, device="cuda")
            ref_i = torch.empty(rows, dtype=torch.int32, device="cuda")
            ws2 = torch.zeros(head.dense_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
            st = head.dense_head_f16(h, e, ref_k, ref_i, None, ws2, rows, hs, vocab, 0,
                                     s.cuda_stream)
            assert st.ok(), st
            s.synchronize()
            ok &= bool(torch.equal(keys, ref_k)) and bool(torch.equal(ids, ref_i))
        ex.close()
        dist.barrier()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_gpu_in_kernel_merge():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=5) for _ in procs)
    assert res == {0: True, 1: True}
