"""Pin the CPU oracle to the reference: every golden fixture was produced by the
reference code itself (tests/golden/make_golden.py).  The oracle runs in fp64;
the fixtures are the reference's fp32 results, so the bound is fp32-level."""
import os

import numpy as np
import pytest
import torch

import oracle
from oracle import composite as oc

TOL = 2e-5  # fp32 reference vs fp64 oracle, relative to max|ref|


def load(golden_dir, name):
    return dict(np.load(os.path.join(golden_dir, name + ".npz")))


@pytest.mark.parametrize("name", ["mm_cfg0", "mm_pad300", "mm_beta0"])
def test_mmscan_matches_reference(golden_dir, name):
    g = load(golden_dir, name)
    beta, alpha = float(g["beta"]), float(g["alpha"])
    y = oracle.mmscan_fwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], beta=beta, alpha=alpha)
    assert oracle.rel_err(y, g["y"]) < TOL
    dx, ddelta, dA, dB, dC, dD, dz, ddb = oracle.mmscan_bwd(
        g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], None, None, False, beta, alpha, g["gy"])
    assert dz is None and ddb is None
    for got, key in ((dx, "dx"), (ddelta, "ddelta"), (dA, "dA"), (dB, "dB"), (dC, "dC"), (dD, "dD")):
        assert oracle.rel_err(got, g[key]) < TOL, key


def test_rows_match_sequential_reference(golden_dir):
    g = load(golden_dir, "mm_seq")
    Bsz, L, ED, N = g["deltaA"].shape
    to_rows = lambda t: np.moveaxis(t, 1, 3).reshape(-1, L)
    back = lambda r: np.moveaxis(r.reshape(Bsz, ED, N, L), 3, 1)
    h = oracle.rows_fwd(to_rows(g["deltaA"]), float(g["beta"]), to_rows(g["u"]))
    assert oracle.rel_err(back(h), g["h"]) < TOL
    da, du = oracle.rows_bwd(to_rows(g["gh"]), to_rows(g["deltaA"]), float(g["beta"]), h)
    assert oracle.rel_err(back(da), g["ddeltaA"]) < TOL
    assert oracle.rel_err(back(du), g["du"]) < TOL


@pytest.mark.parametrize("name", ["pscan_64", "pscan_100"])
def test_pscan_matches_reference(golden_dir, name):
    g = load(golden_dir, name)
    H = oracle.pscan_fwd(g["A"], g["X"])
    assert oracle.rel_err(H, g["H"]) < TOL
    dA, dX = oracle.pscan_bwd(g["A"], H, g["gH"])
    assert oracle.rel_err(dA, g["dA"]) < TOL
    assert oracle.rel_err(dX, g["dX"]) < TOL


def test_scan2_complex_matches_reference(golden_dir):
    g = load(golden_dir, "lin_vec")
    Ms, X = oracle.scan2_fwd(g["M"], g["F"])
    assert oracle.rel_err(Ms, g["Mscan"]) < TOL
    assert oracle.rel_err(X, g["X"]) < TOL
    dM, dF = oracle.scan2_bwd(g["M"], X, g["gX"], Mscan=Ms, gMscan=g["gMscan"])
    assert oracle.rel_err(dM, g["dM"]) < TOL
    assert oracle.rel_err(dF, g["dF"]) < TOL


def test_scan2_real_matches_reference(golden_dir):
    g = load(golden_dir, "lin_pt")
    Ms, X = oracle.scan2_fwd(g["M"][None], g["F"][None])
    assert oracle.rel_err(Ms[0], g["Mscan"]) < TOL
    assert oracle.rel_err(X[0], g["X"]) < TOL
    dM, dF = oracle.scan2_bwd(g["M"][None], X, g["gX"][None])
    assert oracle.rel_err(dM[0], g["dM"]) < TOL
    assert oracle.rel_err(dF[0], g["dF"]) < TOL


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
def test_linoss_apply_matches_reference(golden_dir, disc):
    g = load(golden_dir, "lin_" + disc.lower())
    names = ["A_diag", "B_real", "B_imag", "C_real", "C_imag", "u", "step"]
    ins = oc.to64(*[g[k] for k in names])
    y = oc.linoss_apply(disc, *ins)
    assert oracle.rel_err(y.detach().numpy(), g["y"]) < TOL
    grads = torch.autograd.grad(y, ins, torch.from_numpy(g["gy"]).double())
    for gr, k in zip(grads, names):
        assert oracle.rel_err(gr.numpy(), g["d" + k]) < 5 * TOL, k


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
def test_linoss_layer_matches_reference(golden_dir, disc):
    g = load(golden_dir, "lin_layer_" + disc.lower())
    names = ["u", "A_diag", "B_real", "B_imag", "C_real", "C_imag", "D", "steps"]
    ins = oc.to64(*[g[k] for k in names])
    y = oc.linoss_layer(disc, *ins)
    assert oracle.rel_err(y.detach().numpy(), g["y"]) < TOL
    grads = torch.autograd.grad(y, ins, torch.from_numpy(g["gy"]).double())
    for gr, k in zip(grads, names):
        assert oracle.rel_err(gr.numpy(), g["d" + k]) < 5 * TOL, k


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
def test_mamba_linoss_matches_reference(golden_dir, disc):
    g = load(golden_dir, "mlin_" + disc.lower())
    names = ["A_diag", "B_real", "B_imag", "C_real", "C_imag", "x", "delta"]
    ins = oc.to64(*[g[k] for k in names])
    y = oc.mlinoss_apply(disc, *ins)
    assert oracle.rel_err(y.detach().numpy(), g["y"]) < TOL
    grads = torch.autograd.grad(y, ins, torch.from_numpy(g["gy"]).double(), allow_unused=True)
    for gr, k in zip(grads, names):
        ref = g["d" + k]
        got = np.zeros_like(ref) if gr is None else gr.numpy()
        assert oracle.rel_err(got, ref) < 5 * TOL, k


def test_oracle_f32_variant_close_to_f64(golden_dir):
    g = load(golden_dir, "mm_cfg0")
    y64 = oracle.mmscan_fwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], beta=0.9, alpha=1.0)
    y32 = oracle.mmscan_fwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], beta=0.9, alpha=1.0,
                            prec="f32")
    assert y32.dtype == np.float32
    assert oracle.rel_err(y32, y64) < 1e-5
