"""Segment carries of the momentum scan, on the CPU oracle.

A sequence split into consecutive segments is scanned segment by segment when
each segment receives the state left by the one before it (forward) and the
adjoint pair (a gh, gv) left by the one after it (backward).  Each segment's
effect on an incoming carry is affine with coefficients that a zero-carry pass
over the segment yields (the segment summary):

  forward   h_T = P h_0 + beta Q' v_0 + h^0        v_T = beta^T v_0 + v^0
  backward  lam_0 = P lam_T + lam^0                mu_0 = Q' lam_T + beta^T mu_T + mu^0

with P = prod a_t and Q' = sum_t beta^(t-1) prod_{s>t} a_s over the segment.
These tests pin that algebra (which the sequence-sharded GPU path relies on)
against the unsplit oracle, in fp64.
"""
import numpy as np
import pytest

import oracle

BETA, ALPHA = 0.8, 1.0
TOL = 1e-10


def _inputs(seed, Bsz=2, L=100, Dm=8, N=16, gate=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((Bsz, L, Dm))
    delta = 0.5 * rng.standard_normal((Bsz, L, Dm)) - 2.0
    A = -np.tile(np.arange(1, N + 1, dtype=np.float64), (Dm, 1)) * rng.uniform(0.5, 1.5, (Dm, N))
    B = rng.standard_normal((Bsz, L, N))
    C = rng.standard_normal((Bsz, L, N))
    D = rng.standard_normal(Dm)
    z = rng.standard_normal((Bsz, L, Dm)) if gate else None
    bias = 0.1 * rng.standard_normal(Dm)
    dout = rng.standard_normal((Bsz, L, Dm))
    return dict(x=x, delta=delta, A=A, B=B, C=C, D=D, z=z, bias=bias, dout=dout)


def _seg(t, a, b):
    return None if t is None else t[:, a:b]


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


def _bounds(L, cuts):
    edges = [0] + list(cuts) + [L]
    return list(zip(edges[:-1], edges[1:]))


@pytest.mark.parametrize("cuts", [(37, 77), (1, 2, 99), (50,)])
def test_segments_with_carries_equal_the_whole_sequence(cuts):
    g = _inputs(1)
    args = dict(delta_softplus=True, beta=BETA, alpha=ALPHA)
    y_full, s_full = oracle.mmscan_fwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"],
                                       g["bias"], return_state=True, **args)
    full_g = oracle.mmscan_bwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], g["bias"],
                               True, BETA, ALPHA, g["dout"])
    segs = _bounds(g["x"].shape[1], cuts)
    ys, states, st = [], [], None
    for a, b in segs:
        states.append(st)
        y, st = oracle.mmscan_fwd(_seg(g["x"], a, b), _seg(g["delta"], a, b), g["A"],
                                  _seg(g["B"], a, b), _seg(g["C"], a, b), g["D"], _seg(g["z"], a, b),
                                  g["bias"], state_in=st, return_state=True, **args)
        ys.append(y)
    assert _rel(np.concatenate(ys, 1), y_full) < TOL
    assert _rel(st, s_full) < TOL
    # backward, right to left
    parts, gst = [None] * len(segs), None
    for i in reversed(range(len(segs))):
        a, b = segs[i]
        r = oracle.mmscan_bwd(_seg(g["x"], a, b), _seg(g["delta"], a, b), g["A"], _seg(g["B"], a, b),
                              _seg(g["C"], a, b), g["D"], _seg(g["z"], a, b), g["bias"], True, BETA,
                              ALPHA, _seg(g["dout"], a, b), state_in=states[i], gstate_in=gst,
                              return_gstate=True)
        parts[i], gst = r[:8], r[8]
    names = ["dx", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"]
    for k, name in enumerate(names):
        if name in ("dA", "dD", "ddelta_bias"):
            got = sum(p[k] for p in parts)
        else:
            got = np.concatenate([p[k] for p in parts], 1)
        assert _rel(got, full_g[k]) < TOL, name


def test_segment_summary_is_the_affine_map_of_the_carries():
    g = _inputs(2, L=57)
    rng = np.random.default_rng(5)
    Bsz, L, Dm = g["x"].shape
    N = g["A"].shape[1]
    s_in = rng.standard_normal((Bsz, Dm, 2, N))
    summ = oracle.mmscan_fwd_summary(g["x"], g["delta"], g["A"], g["B"], g["bias"], True, BETA, ALPHA)
    h0, v0, P, Q = summ[:, :, 0], summ[:, :, 1], summ[:, :, 2], summ[:, :, 3]
    _, s_out = oracle.mmscan_fwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], g["bias"],
                                 True, BETA, ALPHA, state_in=s_in, return_state=True)
    assert _rel(s_out[:, :, 0], P * s_in[:, :, 0] + BETA * Q * s_in[:, :, 1] + h0) < TOL
    assert _rel(s_out[:, :, 1], BETA ** L * s_in[:, :, 1] + v0) < TOL
    # the zero-state end state is the forward's own end state
    _, s0 = oracle.mmscan_fwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], g["bias"],
                              True, BETA, ALPHA, return_state=True)
    assert _rel(s0[:, :, 0], h0) < TOL and _rel(s0[:, :, 1], v0) < TOL
    # backward: the same P and Q' map the adjoint carry
    g_in = rng.standard_normal((Bsz, Dm, 2, N))
    bw = lambda gi: oracle.mmscan_bwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"],
                                      g["bias"], True, BETA, ALPHA, g["dout"], state_in=s_in,
                                      gstate_in=gi, return_gstate=True)[8]
    g0, g1 = bw(None), bw(g_in)
    lam, mu = g_in[:, :, 0], g_in[:, :, 1]
    assert _rel(g1[:, :, 0], P * lam + g0[:, :, 0]) < TOL
    assert _rel(g1[:, :, 1], Q * lam + BETA ** L * mu + g0[:, :, 1]) < TOL
