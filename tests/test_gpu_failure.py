"""Failure detection on the GPU without a GPU fault.

The momentum kernels' tile pipelines wait on transaction barriers with a poll
limit; a wait that gives up makes its CTA leave and sets a device flag that
mmb_device_status reports as MMB_ERR_TIMEOUT.  Here the self-test entry point
makes one such wait run out (a barrier armed for bytes that no copy ever
delivers, so nothing asynchronous is outstanding): the status must be
reported once, then cleared, and the context must stay usable for the scans.
"""
import numpy as np
import pytest
import torch

import oracle
from momentummamba_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
MMB_OK, MMB_ERR_TIMEOUT = 0, 7


def test_bounded_wait_reports_timeout_then_clears():
    lib = _lib.load()
    s = _lib.stream_of(torch.empty(1, device=DEV))
    assert lib.mmb_device_status(s) == MMB_OK          # nothing pending before
    assert lib.mmb_selftest_device_wait(256, s) == MMB_OK
    assert lib.mmb_device_status(s) == MMB_ERR_TIMEOUT
    assert lib.mmb_device_status(s) == MMB_OK          # reported once, then cleared

    # the context is still usable: a momentum scan against the fp64 oracle (1e-4)
    from momentummamba_b200 import selective_scan_momentum_fn
    rng = np.random.default_rng(5)
    Bsz, L, Dm, N = 2, 40, 16, 16
    x = rng.standard_normal((Bsz, L, Dm)).astype(np.float32)
    dl = np.log1p(np.exp(0.5 * rng.standard_normal((Bsz, L, Dm)) - 2.0)).astype(np.float32)
    A = -np.tile(np.arange(1, N + 1, dtype=np.float32), (Dm, 1))
    Bm = rng.standard_normal((Bsz, L, N)).astype(np.float32)
    Cm = rng.standard_normal((Bsz, L, N)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(DEV)
    y = selective_scan_momentum_fn(t(x), t(dl), t(A), t(Bm), t(Cm), None, beta=0.7, alpha=1.0)
    yo = oracle.mmscan_fwd(x, dl, A, Bm, Cm, None, None, None, False, 0.7, 1.0)
    assert oracle.rel_err(y.cpu().numpy(), yo) <= 1e-4
    assert lib.mmb_device_status(s) == MMB_OK
