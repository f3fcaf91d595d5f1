"""Shared helpers for the parity tests (host side)."""
from __future__ import annotations

import numpy as np

INVALID = 0xFFFFFFFF
# Acceptance rule: token ids are bit-exact against the FP32 CPU oracle except
# where the oracle's top-2 margin within the allowed set is below 1e-3;
# scores agree within 2e-3 relative.
MARGIN = 1e-3
SCORE_RTOL = 2e-3
SCORE_ATOL = 1e-6


def to_dev(a, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def check_head_parity(gpu_ids, gpu_scores, orc_ids, orc_best, orc_runner_up):
    """Asserts the acceptance rule; returns the number of rows exempted by
    the margin rule."""
    gpu_ids = np.asarray(gpu_ids).astype(np.uint32)
    orc_ids = np.asarray(orc_ids).astype(np.uint32)
    invalid = orc_ids == INVALID
    assert np.array_equal(gpu_ids[invalid], orc_ids[invalid]), "sentinel rows differ"
    valid = ~invalid
    best = np.asarray(orc_best, np.float64)
    ru = np.asarray(orc_runner_up, np.float64)
    nan_rows = valid & np.isnan(best)  # all-NaN rows: lowest id, exact
    assert np.array_equal(gpu_ids[nan_rows], orc_ids[nan_rows]), "all-NaN fallback differs"
    finite = valid & ~np.isnan(best)
    margin = best - ru
    strict = finite & ~(margin < MARGIN)
    bad = np.nonzero(strict & (gpu_ids != orc_ids))[0]
    assert bad.size == 0, (
        f"{bad.size} rows differ with margin >= {MARGIN}: rows {bad[:8]}, "
        f"gpu {gpu_ids[bad[:8]]}, oracle {orc_ids[bad[:8]]}, margin {margin[bad[:8]]}")
    if gpu_scores is not None:
        gs = np.asarray(gpu_scores, np.float64)
        assert np.all(np.isnan(gs[invalid | nan_rows])), "sentinel/NaN rows must report NaN"
        np.testing.assert_allclose(gs[strict], best[strict], rtol=SCORE_RTOL, atol=SCORE_ATOL)
        # a margin-exempt row may report the runner-up's score
        loose = finite & ~strict
        np.testing.assert_allclose(gs[loose], best[loose], rtol=SCORE_RTOL, atol=MARGIN)
    return int((finite & (margin < MARGIN)).sum())


_STREAM = None


def gpu_stream():
    """A dedicated non-blocking CUDA stream (the reference's CudaStream is
    created cudaStreamNonBlocking, src/cuda/cuda_stream.cu:13; the legacy
    default stream has handle 0, which the API rejects as a null stream).
    Inputs are staged with synchronous copies, and results are read after
    torch.cuda.synchronize()."""
    global _STREAM
    import torch

    if _STREAM is None:
        _STREAM = torch.cuda.Stream()
    torch.cuda.synchronize()
    return _STREAM
