"""GPU parity of the momentum selective scan kernels against the CPU oracle
(fp64 arbiter) and the reference's own golden outputs.

Tolerance (stated for every comparison): max|gpu - ref| / max|ref| <= 1e-4 on
the output and on every gradient.
"""
import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-4
DEV = "cuda:0"


def _cuda(a, grad=True):
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(DEV)
    return t.requires_grad_(grad)


def run_gpu(x, delta, A, B, C, D=None, z=None, dbias=None, softplus=False, beta=0.6, alpha=1.0,
            dout=None):
    from momentummamba_b200 import selective_scan_momentum_fn
    ins = {k: (None if v is None else _cuda(v)) for k, v in
           dict(x=x, delta=delta, A=A, B=B, C=C, D=D, z=z, dbias=dbias).items()}
    args = ins
    y = selective_scan_momentum_fn(args["x"], args["delta"], args["A"], args["B"], args["C"],
                                   args["D"], z=args["z"], delta_bias=args["dbias"],
                                   delta_softplus=softplus, beta=beta, alpha=alpha)
    keys = [k for k, v in ins.items() if v is not None]
    grads = torch.autograd.grad(y, [ins[k] for k in keys], _cuda(dout, False))
    torch.cuda.synchronize()
    return y.detach().cpu().numpy(), {k: g.cpu().numpy() for k, g in zip(keys, grads)}


def run_oracle(x, delta, A, B, C, D=None, z=None, dbias=None, softplus=False, beta=0.6, alpha=1.0,
               dout=None):
    y = oracle.mmscan_fwd(x, delta, A, B, C, D, z, dbias, softplus, beta, alpha)
    r = oracle.mmscan_bwd(x, delta, A, B, C, D, z, dbias, softplus, beta, alpha, dout)
    names = ["x", "delta", "A", "B", "C", "D", "z", "dbias"]
    return y, {k: v for k, v in zip(names, r) if v is not None}


def assert_close(got, want, what, tol=TOL):
    err = oracle.rel_err(got, want)
    assert err <= tol, f"{what}: rel err {err:.3e} > {tol}"


def make_inputs(rng, Bsz, L, Dm, N, z=False, bias=False, Dskip=True):
    x = rng.standard_normal((Bsz, L, Dm))
    if bias:
        delta = 0.5 * rng.standard_normal((Bsz, L, Dm)) - 2.0  # raw, softplus in kernel
    else:
        delta = np.log1p(np.exp(0.5 * rng.standard_normal((Bsz, L, Dm)) - 2.0))
    A = -np.tile(np.arange(1, N + 1, dtype=np.float64), (Dm, 1)) * rng.uniform(0.5, 1.5, (Dm, 1))
    B = rng.standard_normal((Bsz, L, N))
    C = rng.standard_normal((Bsz, L, N))
    D = rng.standard_normal(Dm) if Dskip else None
    zz = rng.standard_normal((Bsz, L, Dm)) if z else None
    db = 0.3 * rng.standard_normal(Dm) if bias else None
    dout = rng.standard_normal((Bsz, L, Dm))
    f = lambda a: None if a is None else a.astype(np.float32).astype(np.float64)
    return dict(x=f(x), delta=f(delta), A=f(A), B=f(B), C=f(C), D=f(D), z=f(zz), dbias=f(db),
                dout=f(dout))


def check_case(inp, softplus, beta, alpha, tol=TOL):
    y, g = run_gpu(**inp, softplus=softplus, beta=beta, alpha=alpha)
    yo, go = run_oracle(**inp, softplus=softplus, beta=beta, alpha=alpha)
    assert_close(y, yo, "y", tol)
    for k in go:
        assert_close(g[k], go[k], "d" + k, tol)


@pytest.mark.parametrize("name", ["mm_cfg0", "mm_pad300", "mm_beta0"])
def test_golden_reference_cases(golden_dir, name):
    """The BASELINE operator case (and its edge variants) against the reference's
    own fp32 PScan outputs and against the fp64 oracle."""
    g = dict(np.load(os.path.join(golden_dir, name + ".npz")))
    beta, alpha = float(g["beta"]), float(g["alpha"])
    inp = dict(x=g["x"], delta=g["delta"], A=g["A"], B=g["B"], C=g["C"], D=g["D"], dout=g["gy"])
    y, gr = run_gpu(**inp, beta=beta, alpha=alpha)
    assert_close(y, g["y"], "y vs reference")
    for k in ("x", "delta", "A", "B", "C", "D"):
        assert_close(gr[k], g["d" + k], f"d{k} vs reference")
    yo, go = run_oracle(**inp, beta=beta, alpha=alpha)
    assert_close(y, yo, "y vs oracle")
    for k in go:
        assert_close(gr[k], go[k], f"d{k} vs oracle")


CASES = [
    # (B, L, D, N, z, bias, Dskip, beta, alpha)
    (2, 100, 40, 16, True, True, True, 0.9, 1.0),
    (1, 1, 8, 16, False, False, True, 0.6, 1.0),
    (3, 33, 24, 8, True, False, False, 0.6, 0.5),
    (1, 257, 64, 32, False, True, True, 0.3, 1.0),
    (1, 64, 20, 64, True, True, True, 0.9, 1.0),
    (2, 50, 12, 4, False, False, True, 0.6, 1.0),   # N=4 runs padded to 8
    (2, 70, 16, 12, True, False, True, 0.0, 1.0),   # N=12 runs padded to 16, beta = 0
    (1, 300, 128, 16, True, True, True, 0.95, 2.0),
    # many channels: 4 states per thread (fewer channels run 2 per thread)
    (48, 40, 512, 16, True, True, True, 0.9, 1.0),
    (40, 21, 1000, 8, True, False, True, 0.5, 1.0),
    (20, 33, 520, 32, False, True, True, 0.7, 1.0),
]


@pytest.mark.parametrize("case", CASES, ids=[str(c[:4]) for c in CASES])
def test_random_shapes(case):
    Bsz, L, Dm, N, z, bias, Dskip, beta, alpha = case
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    inp = make_inputs(rng, Bsz, L, Dm, N, z=z, bias=bias, Dskip=Dskip)
    check_case(inp, softplus=bias, beta=beta, alpha=alpha)


def test_strided_views_and_unaligned_rows():
    """B and C as column slices of one projection (the x_proj split of the block)
    and z as a slice of the in_proj output: once with 16-byte aligned row strides
    and once with odd ones (the 4-byte staging path)."""
    from momentummamba_b200 import selective_scan_momentum_fn
    rng = np.random.default_rng(7)
    Bsz, L, Dm, N = 2, 45, 24, 16
    inp = make_inputs(rng, Bsz, L, Dm, N, z=True, bias=True)
    yo, go = run_oracle(**inp, softplus=True, beta=0.8, alpha=1.0)
    for extra in (8, 9):
        off = Dm + (extra - 8)
        proj = torch.zeros(Bsz, L, extra + 2 * N, device=DEV)
        proj[..., extra:extra + N] = _cuda(inp["B"], False)
        proj[..., extra + N:] = _cuda(inp["C"], False)
        xz = torch.zeros(Bsz, L, off + Dm, device=DEV)
        xz[..., off:] = _cuda(inp["z"], False)
        proj.requires_grad_(True)
        xz.requires_grad_(True)
        x, delta, A, D, db = (_cuda(inp[k]) for k in ("x", "delta", "A", "D", "dbias"))
        Bv, Cv, zv = proj[..., extra:extra + N], proj[..., extra + N:], xz[..., off:]
        assert Bv.stride(1) == extra + 2 * N and zv.stride(1) == off + Dm
        y = selective_scan_momentum_fn(x, delta, A, Bv, Cv, D, z=zv, delta_bias=db,
                                       delta_softplus=True, beta=0.8, alpha=1.0)
        gx, gd, gA, gp, gz, gD, gdb = torch.autograd.grad(
            y, [x, delta, A, proj, xz, D, db], _cuda(inp["dout"], False))
        got = dict(x=gx, delta=gd, A=gA, B=gp[..., extra:extra + N], C=gp[..., extra + N:],
                   z=gz[..., off:], D=gD, dbias=gdb)
        assert_close(y.detach().cpu().numpy(), yo, f"y (extra={extra})")
        for k in go:
            assert_close(got[k].cpu().numpy(), go[k], f"d{k} (extra={extra})")


def test_config1_layer_full_size():
    """One MambaMomentum layer's scan at the stack's full size (B=32, L=1024, D=256,
    N=16, z-gate, softplus+bias): outputs and all gradients vs the fp64 oracle."""
    rng = np.random.default_rng(1)
    inp = make_inputs(rng, 32, 1024, 256, 16, z=True, bias=True)
    check_case(inp, softplus=True, beta=0.6, alpha=1.0)


def test_linearity_and_reproducibility():
    """Size-independent properties at a larger size: the backward is linear in
    dout, and the forward is bitwise reproducible."""
    from momentummamba_b200 import selective_scan_momentum_fn
    g = torch.Generator(device=DEV).manual_seed(3)
    Bsz, L, Dm, N = 8, 2048, 512, 16
    x = torch.randn(Bsz, L, Dm, device=DEV, generator=g, requires_grad=True)
    delta = torch.nn.functional.softplus(torch.randn(Bsz, L, Dm, device=DEV, generator=g) - 2)
    delta.requires_grad_(True)
    A = -torch.arange(1, N + 1, device=DEV, dtype=torch.float32).repeat(Dm, 1)
    Bm = torch.randn(Bsz, L, N, device=DEV, generator=g)
    Cm = torch.randn(Bsz, L, N, device=DEV, generator=g)
    y1 = selective_scan_momentum_fn(x, delta, A, Bm, Cm, beta=0.9)
    y2 = selective_scan_momentum_fn(x, delta, A, Bm, Cm, beta=0.9)
    assert torch.equal(y1, y2)
    dout = torch.randn(y1.shape, device=DEV, generator=g)
    gx1, gd1 = torch.autograd.grad(y1, [x, delta], dout)
    gx2, gd2 = torch.autograd.grad(y2, [x, delta], 2.5 * dout)
    assert oracle.rel_err((gx2 / 2.5).cpu().numpy(), gx1.cpu().numpy()) < 1e-6
    assert oracle.rel_err((gd2 / 2.5).cpu().numpy(), gd1.cpu().numpy()) < 1e-6
    assert torch.isfinite(y1).all()


# ---------------------------------------------------------------------------
# row scans and PScan layout
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("R,L,beta", [(300, 256, 0.9), (7, 1, 0.5), (129, 37, 0.0), (64, 1000, 0.6)])
def test_momentum_scan_cuda_rows(R, L, beta):
    from momentummamba_b200.momentum_scan_cuda import momentum_scan_cuda
    from momentummamba_b200.warp_momentum_scan_cuda import warp_momentum_scan_cuda
    rng = np.random.default_rng(R * 1000 + L)
    a = np.exp(-rng.uniform(0, 1, (R, L))).astype(np.float32)
    u = rng.standard_normal((R, L)).astype(np.float32)
    gh = rng.standard_normal((R, L)).astype(np.float32)
    ho = oracle.rows_fwd(a, beta, u)
    dao, duo = oracle.rows_bwd(gh, a, beta, ho)
    for fn in (momentum_scan_cuda, warp_momentum_scan_cuda):
        at, ut = _cuda(a), _cuda(u)
        h = fn(at, beta, ut)
        da, du = torch.autograd.grad(h, [at, ut], _cuda(gh, False))
        assert_close(h.detach().cpu().numpy(), ho, "h")
        assert_close(da.cpu().numpy(), dao, "ddeltaA")
        assert_close(du.cpu().numpy(), duo, "du")
        assert float(da[:, 0].abs().max()) == 0.0


def test_rows_golden_sequential(golden_dir):
    """Reference _sequential_momentum_scan outputs through the block's row path."""
    from momentummamba_b200.mamba_momentum import MambaMomentumBlock, MambaMomentumConfig
    g = dict(np.load(os.path.join(golden_dir, "mm_seq.npz")))
    blk = MambaMomentumBlock(MambaMomentumConfig(d_model=4, n_layers=1, d_state=4)).to(DEV)
    a, u = _cuda(g["deltaA"]), _cuda(g["u"])
    h = blk._sequential_momentum_scan(a, float(g["beta"]), u)
    da, du = torch.autograd.grad(h, [a, u], _cuda(g["gh"], False))
    assert_close(h.detach().cpu().numpy(), g["h"], "h")
    assert_close(da.cpu().numpy(), g["ddeltaA"], "ddeltaA")
    assert_close(du.cpu().numpy(), g["du"], "du")


def test_reference_launcher_api():
    from momentummamba_b200.momentum_scan_cuda import get_momentum_kernel
    k = get_momentum_kernel()
    rng = np.random.default_rng(5)
    a = np.exp(-rng.uniform(0, 1, (40, 64))).astype(np.float32)
    u = rng.standard_normal((40, 64)).astype(np.float32)
    g = rng.standard_normal((40, 64)).astype(np.float32)
    at, ut, gt = (torch.from_numpy(v).to(DEV) for v in (a, u, g))
    h = torch.zeros_like(at)
    k.launch_forward(at, 0.7, ut, h)
    da, du = torch.zeros_like(at), torch.empty(0, device=DEV)
    k.launch_backward(gt, at, 0.7, h, da, du)
    torch.cuda.synchronize()
    ho = oracle.rows_fwd(a, 0.7, u)
    assert_close(h.cpu().numpy(), ho, "h")
    assert_close(da.cpu().numpy(), oracle.rows_bwd(g, a, 0.7, ho)[0], "da")


@pytest.mark.parametrize("name", ["pscan_64", "pscan_100"])
def test_pscan_golden(golden_dir, name):
    from momentummamba_b200.pscan import pscan
    g = dict(np.load(os.path.join(golden_dir, name + ".npz")))
    A, X = _cuda(g["A"]), _cuda(g["X"])
    H = pscan(A, X)
    dA, dX = torch.autograd.grad(H, [A, X], _cuda(g["gH"], False))
    assert_close(H.detach().cpu().numpy(), g["H"], "H")
    assert_close(dA.cpu().numpy(), g["dA"], "dA")
    assert_close(dX.cpu().numpy(), g["dX"], "dX")


def test_pscan_large():
    from momentummamba_b200.pscan import pscan
    rng = np.random.default_rng(9)
    A = np.exp(-rng.uniform(0, 0.2, (3, 301, 40, 16))).astype(np.float32)
    X = rng.standard_normal((3, 301, 40, 16)).astype(np.float32)
    G = rng.standard_normal((3, 301, 40, 16)).astype(np.float32)
    At, Xt = _cuda(A), _cuda(X)
    H = pscan(At, Xt)
    dA, dX = torch.autograd.grad(H, [At, Xt], _cuda(G, False))
    Ho = oracle.pscan_fwd(A, X)
    dAo, dXo = oracle.pscan_bwd(A, Ho, G)
    assert_close(H.detach().cpu().numpy(), Ho, "H")
    assert_close(dA.cpu().numpy(), dAo, "dA")
    assert_close(dX.cpu().numpy(), dXo, "dX")


# ---------------------------------------------------------------------------
# model level
# ---------------------------------------------------------------------------
def test_mamba_momentum_stack_matches_oracle(monkeypatch):
    """Two MambaMomentum layers (fused gate + softplus in the kernel) on the GPU vs
    an fp64 CPU copy of the same module whose scan is the oracle: loss and every
    parameter gradient."""
    from oracle import composite as oc
    import momentummamba_b200.mamba_momentum as mm
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    cfg = mm.MambaMomentumConfig(d_model=32, n_layers=2, dt_rank=4, momentum_beta=0.9)
    gpu = mm.MambaMomentum(cfg).to(DEV)
    cpu = mm.MambaMomentum(cfg).double()
    cpu.load_state_dict(gpu.state_dict())
    x = torch.randn(2, 80, 32)

    out = gpu(x.to(DEV))
    loss = out.pow(2).mean()
    loss.backward()

    def oracle_scan(x, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                    beta=0.6, alpha=1.0):
        return oc.mmscan(x, delta, A, B, C, D, z, delta_bias, delta_softplus, beta, alpha)

    monkeypatch.setattr(mm, "selective_scan_momentum_fn", oracle_scan)
    monkeypatch.setattr(mm, "conv1d_silu", oc.conv1d_silu)
    out_c = cpu(x.double())
    loss_c = out_c.pow(2).mean()
    loss_c.backward()
    assert abs(loss.item() - loss_c.item()) <= TOL * abs(loss_c.item())
    for (n, p), (_, q) in zip(gpu.named_parameters(), cpu.named_parameters()):
        assert_close(p.grad.cpu().numpy(), q.grad.numpy(), "grad " + n)


@pytest.mark.parametrize("mode", ["pscan_sequential", "sequential"])
def test_block_modes_agree(mode):
    """The reference's other pscan_mode paths (materialised tensors on the PScan
    and row kernels) give the fused kernel's result."""
    import momentummamba_b200.mamba_momentum as mm
    torch.manual_seed(1)
    cfg = mm.MambaMomentumConfig(d_model=16, n_layers=1, momentum_beta=0.7)
    fused = mm.MambaMomentum(cfg).to(DEV)
    cfg2 = mm.MambaMomentumConfig(d_model=16, n_layers=1, momentum_beta=0.7, pscan_mode=mode)
    other = mm.MambaMomentum(cfg2).to(DEV)
    other.load_state_dict(fused.state_dict())
    x = torch.randn(2, 50, 16, device=DEV)
    y1 = fused(x)
    y2 = other(x)
    y1.pow(2).sum().backward()
    y2.pow(2).sum().backward()
    assert_close(y1.detach().cpu().numpy(), y2.detach().cpu().numpy(), "y")
    for (n, p), (_, q) in zip(fused.named_parameters(), other.named_parameters()):
        assert_close(p.grad.cpu().numpy(), q.grad.cpu().numpy(), "grad " + n)
