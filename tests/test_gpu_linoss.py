"""GPU parity of the 2x2 (LinOSS) scan kernels against the CPU oracle (fp64)
and the reference's own golden outputs.

Tolerance: max|gpu - ref| / max|ref| <= 1e-4 for outputs and gradients.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from oracle import composite as oc

pytestmark = pytest.mark.gpu

TOL = 1e-4
DEV = "cuda:0"


def close(got, want, what, tol=TOL):
    got = got.detach().cpu().numpy() if isinstance(got, torch.Tensor) else got
    want = want.detach().cpu().numpy() if isinstance(want, torch.Tensor) else want
    err = oracle.rel_err(got, want)
    assert err <= tol, f"{what}: rel err {err:.3e} > {tol}"


def cuda(a, grad=True):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    t = t.to(torch.complex64) if t.is_complex() else t.float()
    return t.requires_grad_(grad)


def load(golden_dir, name):
    return dict(np.load(os.path.join(golden_dir, name + ".npz")))


def rand_M(rng, Bsz, L, P):
    dt = rng.uniform(0.05, 0.55, (Bsz, L, P))
    A = rng.uniform(0, 1, (Bsz, L, P))
    S = 1.0 / (1.0 + dt * dt * A)
    return np.concatenate([1 - dt * dt * A * S, -dt * A * S, dt * S, S], axis=-1).astype(np.float32)


def test_parallel_scan_batched_complex_golden(golden_dir):
    from momentummamba_b200.mamba_linoss import parallel_scan_batched_complex
    g = load(golden_dir, "lin_vec")
    M, Fv = cuda(g["M"]), cuda(g["F"])
    Ms, X = parallel_scan_batched_complex(M, Fv)
    close(Ms, g["Mscan"], "A_scan")
    close(X, g["X"], "b_scan")
    loss = (X.real * cuda(g["gX"].real, False) + X.imag * cuda(g["gX"].imag, False)).sum() + \
        (Ms * cuda(g["gMscan"], False)).sum()
    dM, dF = torch.autograd.grad(loss, [M, Fv])
    close(dM, g["dM"], "dM")
    close(dF, g["dF"], "dF")


def test_parallel_scan_batched_real_golden(golden_dir):
    from momentummamba_b200.LinOSS_pytorch import parallel_scan_batched
    g = load(golden_dir, "lin_pt")
    M, Fv = cuda(g["M"]), cuda(g["F"])
    Ms, X = parallel_scan_batched(M, Fv)
    close(Ms, g["Mscan"], "A_scan")
    close(X, g["X"], "b_scan")
    dM, dF = torch.autograd.grad(X, [M, Fv], cuda(g["gX"], False))
    close(dM, g["dM"], "dM")
    close(dF, g["dF"], "dF")


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
def test_apply_linoss_golden(golden_dir, disc):
    import momentummamba_b200.LinOSS_pytorch as lp
    g = load(golden_dir, "lin_" + disc.lower())
    names = ["A_diag", "B_real", "B_imag", "C_real", "C_imag", "u", "step"]
    ins = [cuda(g[k]) for k in names]
    fn = lp.apply_linoss_im_complex if disc == "IM" else lp.apply_linoss_imex_complex
    y = fn(*ins)
    close(y, g["y"], "y")
    grads = torch.autograd.grad(y, ins, cuda(g["gy"], False))
    for gr, k in zip(grads, names):
        close(gr, g["d" + k], "d" + k)


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
def test_linoss_layer_golden(golden_dir, disc):
    import momentummamba_b200.LinOSS_pytorch as lp
    g = load(golden_dir, "lin_layer_" + disc.lower())
    layer = lp.LinOSSLayer(g["A_diag"].shape[0], g["u"].shape[-1], disc).to(DEV)
    with torch.no_grad():
        for k in ["A_diag", "B_real", "B_imag", "C_real", "C_imag", "D", "steps"]:
            getattr(layer, k).copy_(torch.from_numpy(g[k]))
    u = cuda(g["u"])
    y = layer(u)
    close(y, g["y"], "y")
    params = [layer.A_diag, layer.B_real, layer.B_imag, layer.C_real, layer.C_imag, layer.D,
              layer.steps]
    grads = torch.autograd.grad(y, [u] + params, cuda(g["gy"], False))
    for gr, k in zip(grads, ["u", "A_diag", "B_real", "B_imag", "C_real", "C_imag", "D", "steps"]):
        close(gr, g["d" + k], "d" + k)


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
def test_apply_linoss_vectorized_golden(golden_dir, disc):
    from momentummamba_b200.mamba_linoss import apply_linoss_vectorized
    g = load(golden_dir, "mlin_" + disc.lower())
    names = ["A_diag", "B_real", "B_imag", "C_real", "C_imag", "x", "delta"]
    ins = [cuda(g[k]) for k in names]
    for algo in ("vmap", "optimized", "vectorized"):
        y = apply_linoss_vectorized(disc, *ins, scan_algorithm=algo)
        close(y, g["y"], f"y ({algo})")
    grads = torch.autograd.grad(y, ins, cuda(g["gy"], False), allow_unused=True)
    for gr, k in zip(grads, names):
        gr = torch.zeros_like(ins[names.index(k)]) if gr is None else gr
        close(gr, g["d" + k], "d" + k)


# (1, 1125, 3): 71 chunks of 16 steps (more than two warp rounds of the chunk
# carry scan) and a ragged last chunk of 5 steps
@pytest.mark.parametrize("Bsz,L,P,cplx", [(3, 1000, 40, True), (2, 37, 5, False), (1, 1, 3, True),
                                          (4, 4096, 64, True), (1, 16 * 70 + 5, 3, True),
                                          (1, 16 * 70 + 5, 3, False)])
def test_scan2_random_vs_oracle(Bsz, L, P, cplx):
    from momentummamba_b200.scan2 import scan2
    rng = np.random.default_rng(L * 7 + P)
    M = rand_M(rng, Bsz, L, P)
    if cplx:
        Fv = (rng.standard_normal((Bsz, L, 2 * P)) + 1j * rng.standard_normal((Bsz, L, 2 * P))).astype(np.complex64)
        gX = (rng.standard_normal((Bsz, L, 2 * P)) + 1j * rng.standard_normal((Bsz, L, 2 * P))).astype(np.complex64)
    else:
        Fv = rng.standard_normal((Bsz, L, 2 * P)).astype(np.float32)
        gX = rng.standard_normal((Bsz, L, 2 * P)).astype(np.float32)
    gMs = (0.1 * rng.standard_normal((Bsz, L, 4 * P))).astype(np.float32)
    Mt, Ft = cuda(M), cuda(Fv)
    Ms, X = scan2(Mt, Ft)
    Mso, Xo = oracle.scan2_fwd(M, Fv)
    close(Ms, Mso, "Mscan")
    close(X, Xo, "X")
    if cplx:
        loss = (X.real * cuda(gX.real, False) + X.imag * cuda(gX.imag, False)).sum()
    else:
        loss = (X * cuda(gX, False)).sum()
    loss = loss + (Ms * cuda(gMs, False)).sum()
    dM, dF = torch.autograd.grad(loss, [Mt, Ft])
    dMo, dFo = oracle.scan2_bwd(M, Xo, gX, Mscan=Mso, gMscan=gMs)
    close(dM, dMo, "dM")
    close(dF, dFo, "dF")


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
@pytest.mark.parametrize("Bsz,L,P", [(2, 300, 24), (16, 4096, 256)])
def test_linoss_scan_vs_oracle(disc, Bsz, L, P):
    """The fused LinOSS-layer scan (time-invariant transitions) at the LinOSS
    benchmark size (B=16, L=4096, P=256) and a ragged small case."""
    from momentummamba_b200.scan2 import linoss_scan
    rng = np.random.default_rng(P)
    A = rng.uniform(0, 1, P).astype(np.float32)
    step = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), P)).astype(np.float32)
    Bu = (rng.standard_normal((Bsz, L, P)) + 1j * rng.standard_normal((Bsz, L, P))).astype(np.complex64)
    g = (rng.standard_normal((Bsz, L, P)) + 1j * rng.standard_normal((Bsz, L, P))).astype(np.complex64)
    At, st, Bt = cuda(A), cuda(step), cuda(Bu)
    x2 = linoss_scan(disc, At, st, Bt)
    dA, ds, dBu = torch.autograd.grad((x2.real * cuda(g.real, False) + x2.imag * cuda(g.imag, False)).sum(),
                                      [At, st, Bt])
    # oracle: the same scan through the generic 2x2 restatement, fp64 autograd
    A64, s64, Bu64 = oc.to64(A, step, Bu)
    Mv, f1, f2 = oc._linoss_matrices(disc, A64, s64)
    M = Mv.reshape(1, 1, 4 * P).expand(Bsz, L, 4 * P)
    Fv = torch.cat([f1 * Bu64, f2 * Bu64], dim=-1)
    _, X = oc.scan2(M, Fv)
    x2o = X[..., P:]
    gt = torch.from_numpy(g).to(torch.complex128)
    lo = (x2o.real * gt.real + x2o.imag * gt.imag).sum()
    dAo, dso, dBuo = torch.autograd.grad(lo, [A64, s64, Bu64])
    close(x2, x2o, "x2")
    close(dBu, dBuo, "dBu")
    close(dA, dAo, "dA_diag")
    close(ds, dso, "dstep")


def test_pscan_matrix_ultra_vs_oracle():
    from momentummamba_b200.pscan_optimized import pad_npo2_2x2, pscan_matrix_ultra
    rng = np.random.default_rng(11)
    Bsz, L = 3, 777
    M4 = rand_M(rng, Bsz, L, 1)
    Fv = rng.standard_normal((Bsz, L, 2)).astype(np.float32)
    g = rng.standard_normal((Bsz, L, 2)).astype(np.float32)
    Mt = cuda(M4.reshape(Bsz, L, 2, 2))
    Ft = cuda(Fv)
    X = pscan_matrix_ultra(Mt, Ft)
    _, Xo = oracle.scan2_fwd(M4, Fv)
    close(X, Xo, "F_scan")
    dM, dF = torch.autograd.grad(X, [Mt, Ft], cuda(g, False))
    dMo, dFo = oracle.scan2_bwd(M4, Xo, g)
    close(dM.reshape(Bsz, L, 4), dMo, "dM")
    close(dF, dFo, "dF")
    Mp, Fp = pad_npo2_2x2(Mt.detach(), Ft.detach())
    assert Mp.shape[1] == 1024 and torch.equal(Mp[:, L:], torch.eye(2, device=DEV).expand(Bsz, 1024 - L, 2, 2))


def test_mamba_linoss_model_runs_and_matches_modes():
    import momentummamba_b200.mamba_linoss as ml
    torch.manual_seed(0)
    m = ml.create_mamba_linoss_fast(d_model=16, n_layer=2).to(DEV)
    x = torch.randn(2, 70, 16, device=DEV)
    y = m(x)
    y.pow(2).mean().backward()
    assert torch.isfinite(y).all()
    assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
@pytest.mark.parametrize("Bsz,L,P,ED", [(2, 37, 20, 6), (3, 300, 64, 8), (2, 1000, 256, 4),
                                        (1, 8, 33, 2)])
def test_selective_linoss_fused_vs_oracle(disc, Bsz, L, P, ED):
    """apply_linoss_vectorized on the fused selective-LinOSS kernels (transitions
    built per step, output contracted in-kernel) vs the fp64 restatement, with
    B and C as column slices of one projection, as the block produces them."""
    from momentummamba_b200.mamba_linoss import apply_linoss_vectorized
    rng = np.random.default_rng(L + P)
    r = 3
    proj = rng.standard_normal((Bsz, L, r + 4 * P)) / np.sqrt(P)
    A = np.exp(rng.uniform(-1.0, 1.0, P))
    delta = np.log1p(np.exp(rng.standard_normal((Bsz, L, ED)) - 1.0))
    x = rng.standard_normal((Bsz, L, ED))
    gy = rng.standard_normal((Bsz, L, ED))
    projt, At, dt_ = cuda(proj), cuda(A), cuda(delta)
    parts = torch.split(projt, [r, P, P, P, P], dim=-1)
    y = apply_linoss_vectorized(disc, At, parts[1], parts[2], parts[3], parts[4], cuda(x, False), dt_,
                                scan_algorithm="vectorized")
    dproj, dA, dd = torch.autograd.grad(y, [projt, At, dt_], cuda(gy, False))
    p64, A64, d64 = (torch.from_numpy(a).double().requires_grad_() for a in (proj, A, delta))
    q = torch.split(p64, [r, P, P, P, P], dim=-1)
    yo = oc.mlinoss_apply(disc, A64, q[1], q[2], q[3], q[4], torch.from_numpy(x).double(), d64)
    dpo, dAo, ddo = torch.autograd.grad(yo, [p64, A64, d64], torch.from_numpy(gy).double())
    close(y, yo, "y")
    close(dproj, dpo, "d(B, C)")
    close(dA, dAo, "dA_diag")
    close(dd, ddo, "ddelta")


def _layer_fp64(disc, A_diag, steps, B_re, B_im, C_re, C_im, D, u):
    """LinOSSLayer.forward restated in float64 with a sequential scan
    (LinOSS_pytorch.py:153-239, 258-312): the arbiter for the tensor-core path."""
    A = torch.relu(A_diag)
    s = torch.sigmoid(steps)
    Bu = torch.complex(u @ B_re.t(), u @ B_im.t())                 # (B, L, P)
    if disc == "IM":
        S = 1.0 / (1.0 + s ** 2 * A)
        m11, m12, m21, m22 = 1.0 - s ** 2 * A * S, -s * A * S, s * S, S
        F1, F2 = m11 * Bu * s, m21 * Bu * s
    else:
        m11, m12, m21, m22 = torch.ones_like(A), -s * A, s, 1.0 - s ** 2 * A
        F1, F2 = Bu * s, Bu * s ** 2
    x1 = torch.zeros_like(Bu[:, 0])
    x2 = torch.zeros_like(Bu[:, 0])
    outs = []
    for t in range(u.shape[1]):
        x1, x2 = m11 * x1 + m12 * x2 + F1[:, t], m21 * x1 + m22 * x2 + F2[:, t]
        outs.append(x2)
    X2 = torch.stack(outs, 1)
    return X2.real @ C_re.t() - X2.imag @ C_im.t() + u * D


@pytest.mark.parametrize("disc", ["IM", "IMEX"])
def test_linoss_layer_tensor_cores_vs_fp64(disc):
    """The whole layer (GEMMs on tcgen05 + scan) at H=128, P=256 over 1024 steps,
    forward and every gradient, against float64.  Tolerance 1e-4 (max-normalised)."""
    import momentummamba_b200.LinOSS_pytorch as lp
    torch.manual_seed(7)
    layer = lp.LinOSSLayer(256, 128, disc).to(DEV)
    u = torch.randn(2, 1024, 128, device=DEV, requires_grad=True)
    y = layer(u)
    gy = torch.randn_like(y)
    params = [layer.A_diag, layer.B_real, layer.B_imag, layer.C_real, layer.C_imag, layer.D,
              layer.steps]
    grads = torch.autograd.grad(y, [u] + params, gy)
    ref_in = [p.detach().double().requires_grad_() for p in params]
    u64 = u.detach().double().requires_grad_()
    A_diag, B_re, B_im, C_re, C_im, D, steps = ref_in
    yr = _layer_fp64(disc, A_diag, steps, B_re, B_im, C_re, C_im, D, u64)
    gref = torch.autograd.grad(yr, [u64] + ref_in, gy.double())
    close(y, yr.detach().cpu().numpy(), "y")
    for g, r, k in zip(grads, gref, ["u", "A_diag", "B_real", "B_imag", "C_real", "C_imag", "D",
                                     "steps"]):
        close(g, r.cpu().numpy(), "d" + k)
