"""The allocation-free ragged head (mf_head_restricted_csr_f16_noalloc).

Some callers of this library may not allocate device memory — code running
inside a host callback, under an allocator that is not allowed to grow, or
in a runtime that only hands out its own input and output buffers.  For them
the library keeps a fixed scratch array per GPU instead of asking for a
workspace.  This test calls that entry point through the C-ABI twice in a
row and checks it against the workspace entry point on the same inputs
(same kernel, so token ids are identical and scores agree within the
parity tolerance used elsewhere) and against the FP32 CPU oracle under
the acceptance rule of the other parity tests.  It lives in its own file, collected last,
and also passes when run alone in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import SCORE_ATOL, SCORE_RTOL, check_head_parity, gpu_stream, to_dev

pytestmark = pytest.mark.gpu


def _run(fn, *args):
    st = fn(*args)
    assert st.ok(), st


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    import torch

    from market_sim_b200 import head, synth
    from oracle import oracle as O

    vocab = 49_152
    emb = synth.embedding(4711, vocab=vocab)
    e_dev = to_dev(emb)
    for call, (seed, rows) in enumerate([(11, 256), (12, 97)]):  # two calls in a row
        hid = to_dev(synth.hidden_states(seed, rows))
        off, ids = synth.ragged_batch(seed, rows=rows, kmax=4096, vocab=vocab)
        off_d, ids_d = to_dev(off), to_dev(ids)
        ref_ids = torch.empty(rows, dtype=torch.int32, device="cuda")
        ref_sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        ws = torch.zeros(head.head_workspace_bytes(rows), dtype=torch.uint8, device="cuda")
        s = gpu_stream()
        _run(head.restricted_output_head_csr_f16, hid, e_dev, off_d, ids_d, ref_ids, ref_sc, ws,
             rows, 576, vocab, s)
        got_ids = torch.empty(rows, dtype=torch.int32, device="cuda")
        got_sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        _run(head.restricted_output_head_csr_f16_noalloc, hid, e_dev, off_d, ids_d, got_ids,
             got_sc, rows, 576, vocab, s)
        torch.cuda.synchronize()
        assert np.array_equal(got_ids.cpu().numpy(), ref_ids.cpu().numpy()), f"call {call}"
        np.testing.assert_allclose(got_sc.cpu().numpy(), ref_sc.cpu().numpy(), rtol=SCORE_RTOL,
                                   atol=SCORE_ATOL)
        o_ids, o_best, o_ru = O.restricted_head_csr(hid.cpu().numpy(), emb, off, ids)
        check_head_parity(got_ids.cpu().numpy().view(np.uint32), got_sc.cpu().numpy(), o_ids,
                          o_best, o_ru)


def test_noalloc_rejects_oversized_batches(cuda):
    from market_sim_b200 import head
    from market_sim_b200._lib import lib

    fake = [ctypes.c_void_p(0x10000 * (i + 1)) for i in range(6)]
    rows = head.NOALLOC_MAX_ROWS + 1
    st = lib.mf_head_restricted_csr_f16_noalloc(fake[0], rows * 576 * 2, fake[1], 49_152 * 576 * 2,
                                                fake[2], (rows + 1) * 4, fake[3], 40, fake[4],
                                                rows * 4, fake[5], rows * 4, rows, 576, 49_152,
                                                ctypes.c_void_p(int(gpu_stream().cuda_stream)))
    assert st.code == head.ErrorCode.resource_limit


def test_noalloc_rejected_call_leaves_scratch_alone(cuda):
    """A call that fails validation must not touch the shared scratch: a
    rejected call between two good calls changes nothing."""
    import torch

    from market_sim_b200 import head, synth

    vocab = 8192
    rows = 64
    e_dev = to_dev(synth.embedding(99, vocab=vocab))
    hid = to_dev(synth.hidden_states(98, rows))
    off, ids = synth.ragged_batch(97, rows=rows, kmax=512, vocab=vocab)
    off_d, ids_d = to_dev(off), to_dev(ids)
    s = gpu_stream()
    first = torch.empty(rows, dtype=torch.int32, device="cuda")
    again = torch.empty(rows, dtype=torch.int32, device="cuda")
    _run(head.restricted_output_head_csr_f16_noalloc, hid, e_dev, off_d, ids_d, first, None,
         rows, 576, vocab, s)
    # wrong vocabulary size for the embedding: rejected before any device work
    st = head.restricted_output_head_csr_f16_noalloc(hid, e_dev, off_d, ids_d, again, None, rows,
                                                     576, vocab + 1, s)
    assert st.code == head.ErrorCode.invalid_argument
    _run(head.restricted_output_head_csr_f16_noalloc, hid, e_dev, off_d, ids_d, again, None,
         rows, 576, vocab, s)
    torch.cuda.synchronize()
    assert np.array_equal(first.cpu().numpy(), again.cpu().numpy())
