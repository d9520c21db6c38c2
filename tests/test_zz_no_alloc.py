"""The no-allocation 2x2 scan forward (mmb_scan2_fwd_noalloc) against the
allocating entry point (mmb_scan2_fwd), through the C ABI.

mmb_scan2_fwd_noalloc exists for callers that cannot give the library device
memory at call time (a host framework that owns all device memory, or a path
where a cudaMalloc and its possible device-wide synchronisation is not
acceptable).  Its scratch is one fixed array per device that every call reuses,
so the test makes two calls in a row with different problems: the second call
must not depend on what the first one left in the array.  It also covers the
case where the array forces fewer chunks than the allocating entry point uses,
and the size limit.

This file is collected last on purpose, so that a run stopping at the first
failure has already run every other test.
"""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

import oracle
from momentummamba_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 1e-4
DEV = "cuda:0"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _scratch_floats():
    """MMB_SCAN2_NOALLOC_SCRATCH_FLOATS as the header defines it."""
    src = open(os.path.join(ROOT, "include", "momentum_scan_b200.h")).read()
    m = re.search(r"#define\s+MMB_SCAN2_NOALLOC_SCRATCH_FLOATS\s+\(1 << (\d+)\)", src)
    assert m, "MMB_SCAN2_NOALLOC_SCRATCH_FLOATS not found in the header"
    return 1 << int(m.group(1))


SCRATCH_FLOATS = _scratch_floats()


def _noalloc(lib):
    fn = lib.mmb_scan2_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int64] * 3 + [ctypes.c_int32] + [ctypes.c_void_p] * 5
    return fn


def _inputs(seed, Bsz, L, P, cplx):
    g = torch.Generator(device=DEV).manual_seed(seed)
    dt = torch.rand(Bsz, L, P, device=DEV, generator=g) * 0.5 + 0.05
    A = torch.rand(Bsz, L, P, device=DEV, generator=g)
    S = 1.0 / (1.0 + dt * dt * A)
    M = torch.cat([1 - dt * dt * A * S, -dt * A * S, dt * S, S], dim=-1).contiguous()
    nc = 2 if cplx else 1
    F = torch.randn(Bsz, L, 2 * P, nc, device=DEV, generator=g).contiguous()
    return M, F


def _rel(a, b):
    return float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("order", ["large_first", "small_first"])
def test_noalloc_matches_allocating_entry_point(order):
    lib = _lib.load()
    fn = _noalloc(lib)
    P_ = _lib.ptr
    cases = [(8, 2048, 256, True, True),    # chunk count capped by the fixed scratch
             (2, 333, 17, False, False),    # ragged, real, no running product
             # batch * P = 65536 chains: the scratch holds one chunk, so every chain
             # runs its whole (ragged) length as one chunk
             (1, 37, SCRATCH_FLOATS // 16, False, False)]
    if order == "small_first":
        cases = cases[::-1]
    for seed, (Bsz, L, P, cplx, want_ms) in enumerate(cases):
        M, F = _inputs(seed + 1, Bsz, L, P, cplx)
        stream = _lib.stream_of(M)
        X = torch.full_like(F, float("nan"))
        Ms = torch.full_like(M, float("nan")) if want_ms else None
        st = fn(Bsz, L, P, int(cplx), P_(M), P_(F), P_(Ms), P_(X), stream)
        assert st == 0, lib.mmb_status_string(st)
        # the allocating entry point with its own workspace
        work = torch.empty(lib.mmb_scan2_work_floats(Bsz, L, P, int(cplx)), device=DEV)
        Xr = torch.empty_like(F)
        Msr = torch.empty_like(M) if want_ms else None
        st = lib.mmb_scan2_fwd(Bsz, L, P, int(cplx), P_(M), P_(F), P_(Msr), P_(Xr), P_(work),
                               stream)
        assert st == 0, lib.mmb_status_string(st)
        torch.cuda.synchronize()
        assert torch.isfinite(X).all()
        assert _rel(X, Xr) <= TOL
        if want_ms:
            assert _rel(Ms, Msr) <= TOL
        if Bsz * L * P <= 1 << 16:  # small enough for the fp64 CPU oracle as well
            Fo = F.cpu().numpy()
            Fo = Fo[..., 0] + 1j * Fo[..., 1] if cplx else Fo[..., 0]
            _, Xo = oracle.scan2_fwd(M.cpu().numpy(), Fo)
            Xg = X.cpu().numpy()
            Xg = Xg[..., 0] + 1j * Xg[..., 1] if cplx else Xg[..., 0]
            assert oracle.rel_err(Xg, Xo) <= TOL


def test_noalloc_rejects_problems_beyond_the_scratch():
    lib = _lib.load()
    fn = _noalloc(lib)
    M, F = _inputs(0, 1, 4, 4, False)
    X = torch.empty_like(F)
    # 16 * batch * P floats must fit the fixed array
    too_many_chains = SCRATCH_FLOATS // 16 + 1
    st = fn(1, 4, too_many_chains, 0, _lib.ptr(M), _lib.ptr(F), None, _lib.ptr(X),
            _lib.stream_of(M))
    assert st == 2  # MMB_ERR_SHAPE
    st = fn(1, 4, 4, 0, _lib.ptr(M), _lib.ptr(F), None, _lib.ptr(X), _lib.stream_of(M))
    assert st == 0
    torch.cuda.synchronize()


def test_no_device_wait_gave_up():
    """After everything above ran, no bounded device-side wait (the TMA tile
    pipelines' transaction barriers) reported a timeout."""
    lib = _lib.load()
    assert lib.mmb_device_status(_lib.stream_of(torch.empty(1, device=DEV))) == 0
