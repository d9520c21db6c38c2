"""CPU oracle for the momentum selective scan and the LinOSS 2x2 scan.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import this package, and only as the checker
(or, for the baseline, as the thing timed on the host cores).  The product
package ``momentummamba_b200`` never imports it and has no CPU fallback.

The arithmetic lives in ``scan_oracle.c`` (a sequential restatement of the
reference recurrences, one OpenMP thread per independent chain); this module
loads the shared library with ctypes and wraps it with numpy.  ``prec='f64'``
selects the double-precision arbiter, ``prec='f32'`` the fp32 restatement that
mirrors the reference's own arithmetic.

Parity pin: ``tests/golden/make_golden.py`` ran the reference itself (its
PScan path and its LinOSS scans) on seeded inputs; ``tests/test_oracle_golden.py``
checks this oracle against those fixtures.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_i64 = ctypes.c_int64
_ptr = ctypes.c_void_p


def build(force: bool = False) -> str:
    """Compile scan_oracle.c with the Makefile beside it; returns the .so path."""
    src = [os.path.join(_HERE, f) for f in ("scan_oracle.c", "scan_oracle_impl.h")]
    stale = (not os.path.exists(_LIB_PATH)) or any(
        os.path.getmtime(s) > os.path.getmtime(_LIB_PATH) for s in src)
    if force or stale:
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        for sfx in ("f64", "f32"):
            getattr(lib, f"orc_mmscan_fwd_{sfx}").argtypes = (
                [_i64] * 4 + [_ptr] * 8 + [ctypes.c_int, ctypes.c_double, ctypes.c_double]
                + [_ptr] * 4)
            getattr(lib, f"orc_mmscan_fwd_summary_{sfx}").argtypes = (
                [_i64] * 4 + [_ptr] * 5 + [ctypes.c_int, ctypes.c_double, ctypes.c_double, _ptr])
            getattr(lib, f"orc_mmscan_bwd_{sfx}").argtypes = (
                [_i64] * 4 + [_ptr] * 8 + [ctypes.c_int, ctypes.c_double, ctypes.c_double]
                + [_ptr] * 12)
            getattr(lib, f"orc_rows_fwd_{sfx}").argtypes = [
                _i64, _i64, _ptr, ctypes.c_double, _ptr, _ptr, _ptr]
            getattr(lib, f"orc_rows_bwd_{sfx}").argtypes = [
                _i64, _i64, _ptr, _ptr, ctypes.c_double, _ptr, _ptr, _ptr]
            getattr(lib, f"orc_scan2_fwd_{sfx}").argtypes = [
                _i64, _i64, _i64, _ptr, _ptr, ctypes.c_int, _ptr, _ptr]
            getattr(lib, f"orc_scan2_bwd_{sfx}").argtypes = [
                _i64, _i64, _i64, _ptr, _ptr, ctypes.c_int, _ptr, _ptr, _ptr, _ptr, _ptr]
        lib.orc_num_threads.restype = ctypes.c_int
        lib.orc_set_num_threads.argtypes = [ctypes.c_int]
        _lib = lib
    return _lib


def num_threads() -> int:
    return _load().orc_num_threads()


def set_num_threads(n: int) -> None:
    _load().orc_set_num_threads(int(n))


def _dt(prec: str):
    if prec not in ("f64", "f32"):
        raise ValueError(f"prec must be 'f64' or 'f32', got {prec!r}")
    return np.float64 if prec == "f64" else np.float32


def _c(a, dt):
    """Contiguous array of dtype dt, or None."""
    if a is None:
        return None
    return np.ascontiguousarray(np.asarray(a), dtype=dt)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------------------
# momentum selective scan  (mamba_momentum.py:256-323 + gating :227-229)
# ---------------------------------------------------------------------------
def mmscan_fwd(x, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
               beta=0.6, alpha=1.0, prec="f64", return_ypre=False, state_in=None,
               return_state=False):
    """y = selective momentum scan; shapes x/delta/z (Bsz,L,Dm), A (Dm,N), B/C (Bsz,L,N).

    state_in (Bsz, Dm, 2, N) = (h, v) before the first step (zeros when None);
    return_state adds the state after the last step, same layout."""
    dt = _dt(prec)
    x, delta, A, B, C = (_c(t, dt) for t in (x, delta, A, B, C))
    D, z, delta_bias, state_in = _c(D, dt), _c(z, dt), _c(delta_bias, dt), _c(state_in, dt)
    Bsz, L, Dm = x.shape
    N = A.shape[1]
    out = np.empty_like(x)
    ypre = np.empty_like(x) if return_ypre else None
    state_out = np.empty((Bsz, Dm, 2, N), dt) if return_state else None
    getattr(_load(), f"orc_mmscan_fwd_{prec}")(
        Bsz, L, Dm, N, _p(x), _p(delta), _p(A), _p(B), _p(C), _p(D), _p(z), _p(delta_bias),
        int(bool(delta_softplus)), float(beta), float(alpha), _p(out), _p(ypre),
        _p(state_in), _p(state_out))
    res = (out,) + ((ypre,) if return_ypre else ()) + ((state_out,) if return_state else ())
    return res if len(res) > 1 else out


def mmscan_fwd_summary(x, delta, A, B, delta_bias=None, delta_softplus=False, beta=0.6,
                       alpha=1.0, prec="f64"):
    """Segment summary (Bsz, Dm, 4, N) = [h^0 | v^0 | P | Q']: the segment's end state
    from a zero state and its transition, h_T = P h_0 + beta Q' v_0 + h^0,
    v_T = beta^T v_0 + v^0."""
    dt = _dt(prec)
    x, delta, A, B = (_c(t, dt) for t in (x, delta, A, B))
    delta_bias = _c(delta_bias, dt)
    Bsz, L, Dm = x.shape
    N = A.shape[1]
    summ = np.empty((Bsz, Dm, 4, N), dt)
    getattr(_load(), f"orc_mmscan_fwd_summary_{prec}")(
        Bsz, L, Dm, N, _p(x), _p(delta), _p(A), _p(B), _p(delta_bias),
        int(bool(delta_softplus)), float(beta), float(alpha), _p(summ))
    return summ


def mmscan_bwd(x, delta, A, B, C, D, z, delta_bias, delta_softplus, beta, alpha, dout,
               prec="f64", state_in=None, gstate_in=None, return_gstate=False):
    """Gradients (dx, ddelta, dA, dB, dC, dD, dz, ddelta_bias); absent inputs give None.

    For one segment of a split sequence: state_in as given to the forward,
    gstate_in (Bsz, Dm, 2, N) = (a gh, gv) arriving from the step after the
    segment; return_gstate appends the same pair leaving its first step."""
    dt = _dt(prec)
    x, delta, A, B, C, dout = (_c(t, dt) for t in (x, delta, A, B, C, dout))
    D, z, delta_bias = _c(D, dt), _c(z, dt), _c(delta_bias, dt)
    state_in, gstate_in = _c(state_in, dt), _c(gstate_in, dt)
    Bsz, L, Dm = x.shape
    N = A.shape[1]
    dx, ddelta = np.empty_like(x), np.empty_like(x)
    dA = np.empty_like(A)
    dB, dC = np.empty_like(B), np.empty_like(C)
    dD = np.empty((Dm,), dt) if D is not None else None
    dz = np.empty_like(x) if z is not None else None
    ddb = np.empty((Dm,), dt) if delta_bias is not None else None
    gout = np.empty((Bsz, Dm, 2, N), dt) if return_gstate else None
    getattr(_load(), f"orc_mmscan_bwd_{prec}")(
        Bsz, L, Dm, N, _p(x), _p(delta), _p(A), _p(B), _p(C), _p(D), _p(z), _p(delta_bias),
        int(bool(delta_softplus)), float(beta), float(alpha), _p(dout),
        _p(dx), _p(ddelta), _p(dA), _p(dB), _p(dC), _p(dD), _p(dz), _p(ddb),
        _p(state_in), _p(gstate_in), _p(gout))
    res = (dx, ddelta, dA, dB, dC, dD, dz, ddb)
    return res + (gout,) if return_gstate else res


# ---------------------------------------------------------------------------
# row scans: momentum_scan_cuda (momentum_scan_cuda.py:22-87) and PScan (pscan.py)
# ---------------------------------------------------------------------------
def rows_fwd(a, beta, u, prec="f64", return_v=False):
    """(R, L) rows: v = beta*v + u ; h = a*h + v.  Returns h (and v)."""
    dt = _dt(prec)
    a, u = _c(a, dt), _c(u, dt)
    R, L = a.shape
    h = np.empty_like(a)
    v = np.empty_like(a) if return_v else None
    getattr(_load(), f"orc_rows_fwd_{prec}")(R, L, _p(a), float(beta), _p(u), _p(h), _p(v))
    return (h, v) if return_v else h


def rows_bwd(g, a, beta, h, prec="f64"):
    """Adjoint of rows_fwd: returns (da, du); da is zero at t = 0."""
    dt = _dt(prec)
    g, a, h = _c(g, dt), _c(a, dt), _c(h, dt)
    R, L = a.shape
    da, du = np.empty_like(a), np.empty_like(a)
    getattr(_load(), f"orc_rows_bwd_{prec}")(R, L, _p(g), _p(a), float(beta), _p(h), _p(da), _p(du))
    return da, du


def pscan_fwd(A, X, prec="f64"):
    """PScan semantics (pscan.py:160-194): H_t = A_t*H_{t-1} + X_t along dim 1 of (B, L, ...)."""
    A = np.asarray(A)
    shp = A.shape
    Bsz, L = shp[0], shp[1]
    a = np.moveaxis(np.asarray(A).reshape(Bsz, L, -1), 1, 2).reshape(-1, L)
    x = np.moveaxis(np.asarray(X).reshape(Bsz, L, -1), 1, 2).reshape(-1, L)
    h = rows_fwd(a, 0.0, x, prec)
    return np.moveaxis(h.reshape(Bsz, -1, L), 2, 1).reshape(shp)


def pscan_bwd(A, H, G, prec="f64"):
    """PScan backward (pscan.py:197-232): returns (gradA, gradX)."""
    A = np.asarray(A)
    shp = A.shape
    Bsz, L = shp[0], shp[1]

    def rows(t):
        return np.moveaxis(np.asarray(t).reshape(Bsz, L, -1), 1, 2).reshape(-1, L)

    da, du = rows_bwd(rows(G), rows(A), 0.0, rows(H), prec)

    def back(r):
        return np.moveaxis(r.reshape(Bsz, -1, L), 2, 1).reshape(shp)

    return back(da), back(du)


# ---------------------------------------------------------------------------
# 2x2 scan (mamba_linoss.py:336-415 / :561-605, LinOSS_pytorch.py:53-132)
# ---------------------------------------------------------------------------
def _as_pairs(F, dt):
    F = np.asarray(F)
    if np.iscomplexobj(F):
        return np.ascontiguousarray(np.stack([F.real, F.imag], axis=-1), dtype=dt), True
    return np.ascontiguousarray(F, dtype=dt), False


def _from_pairs(a, cplx):
    return a[..., 0] + 1j * a[..., 1] if cplx else a


def scan2_fwd(M, F, prec="f64", return_mscan=True):
    """x_t = M_t x_{t-1} + F_t.  M (B, L, 4P) real, F (B, L, 2P) real or complex.
    Returns (Mscan, X) like parallel_scan_batched_complex."""
    dt = _dt(prec)
    M = _c(M, dt)
    Fp, cplx = _as_pairs(F, dt)
    Bsz, L, P4 = M.shape
    P = P4 // 4
    X = np.empty_like(Fp)
    Ms = np.empty_like(M) if return_mscan else None
    getattr(_load(), f"orc_scan2_fwd_{prec}")(Bsz, L, P, _p(M), _p(Fp), int(cplx), _p(Ms), _p(X))
    return Ms, _from_pairs(X, cplx)


def scan2_bwd(M, X, gX, Mscan=None, gMscan=None, prec="f64"):
    """Adjoint of scan2_fwd.  Returns (dM, dF); dF is complex when X is."""
    dt = _dt(prec)
    M = _c(M, dt)
    Xp, cplx = _as_pairs(X, dt)
    gXp = None
    if gX is not None:
        gXp, _ = _as_pairs(gX if not cplx else np.asarray(gX, dtype=np.complex128), dt)
    Ms = _c(Mscan, dt)
    gMs = _c(gMscan, dt)
    Bsz, L, P4 = M.shape
    P = P4 // 4
    dM = np.empty_like(M)
    dF = np.empty_like(Xp)
    getattr(_load(), f"orc_scan2_bwd_{prec}")(Bsz, L, P, _p(M), _p(Xp), int(cplx), _p(gXp),
                                              _p(Ms), _p(gMs), _p(dM), _p(dF))
    return dM, _from_pairs(dF, cplx)


def rel_err(a, b) -> float:
    """max|a - b| / max|b| (the parity metric used throughout the tests)."""
    a = np.asarray(a, dtype=np.complex128 if np.iscomplexobj(a) or np.iscomplexobj(b) else np.float64)
    b = np.asarray(b, dtype=a.dtype)
    den = float(np.max(np.abs(b))) if b.size else 0.0
    num = float(np.max(np.abs(a - b))) if a.size else 0.0
    if den == 0.0:
        return num
    return num / den
