"""GPU parity of the block's producer (causal depthwise conv1d + SiLU) and the
decode-step kernels against the fp64 restatements in oracle/composite.py (which
tests/test_oracle_block.py pins to the reference's own block), and of the
block itself against the reference's golden forward/backward and decode steps.

Tolerance: max|gpu - ref| / max|ref| <= 1e-4 for every output and gradient.
"""
import os

import numpy as np
import pytest
import torch

from oracle import composite as oc

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 1e-4


def rel(a, b):
    a = a.detach().double().cpu() if isinstance(a, torch.Tensor) else torch.from_numpy(a).double()
    b = b.detach().double().cpu() if isinstance(b, torch.Tensor) else torch.from_numpy(b).double()
    return float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("Bsz,L,D,W,bias,strided,state", [
    (2, 37, 64, 4, True, False, False),
    (3, 300, 200, 4, True, True, True),   # ragged channels, a column slice of xz, a state
    (1, 1, 32, 4, False, False, True),
    (2, 64, 128, 2, True, False, False),
    (2, 129, 96, 8, True, True, False),
    (1, 65, 48, 3, False, False, True),
])
def test_conv1d_silu_forward_backward(Bsz, L, D, W, bias, strided, state):
    from momentummamba_b200.conv import conv1d_silu
    g = torch.Generator().manual_seed(L * 7 + D)
    xz = torch.randn(Bsz, L, 2 * D, generator=g, dtype=torch.float64)
    x64 = xz[..., :D] if strided else xz[..., :D].contiguous()
    w64 = 0.5 * torch.randn(D, 1, W, generator=g, dtype=torch.float64)
    b64 = 0.1 * torch.randn(D, generator=g, dtype=torch.float64) if bias else None
    s64 = torch.randn(Bsz, D, W - 1, generator=g, dtype=torch.float64) if state else None
    dout = torch.randn(Bsz, L, D, generator=g, dtype=torch.float64)
    # oracle
    xo, wo = x64.clone().requires_grad_(), w64.clone().requires_grad_()
    bo = None if b64 is None else b64.clone().requires_grad_()
    yo = oc.conv1d_silu(xo, wo, bo, s64)
    go = torch.autograd.grad(yo, [xo, wo] + ([bo] if bo is not None else []), dout)
    # GPU
    xg = (xz.float().to(DEV)[..., :D] if strided else x64.float().to(DEV)).requires_grad_()
    wg = w64.float().to(DEV).requires_grad_()
    bg = None if b64 is None else b64.float().to(DEV).requires_grad_()
    sg = None if s64 is None else s64.float().to(DEV)
    yg = conv1d_silu(xg, wg, bg, sg)
    gg = torch.autograd.grad(yg, [xg, wg] + ([bg] if bg is not None else []), dout.float().to(DEV))
    assert rel(yg, yo) <= TOL
    for name, a, b in zip(["dx", "dweight", "dbias"], gg, go):
        assert rel(a, b) <= TOL, f"{name} {rel(a, b):.2e}"


def test_prefill_then_decode_equals_the_sequence():
    """conv1d_silu_state + conv1d_step, and forward(state_out) + mmscan_step, give
    the same outputs as running the whole sequence at once."""
    from momentummamba_b200.conv import conv1d_silu, conv1d_silu_state, conv1d_step, mmscan_step
    from momentummamba_b200.selective_scan import ScanCall
    torch.manual_seed(3)
    Bsz, L, T, D, N, W = 2, 45, 5, 64, 16, 4
    xin = torch.randn(Bsz, L + T, D, device=DEV)
    w = 0.5 * torch.randn(D, 1, W, device=DEV)
    b = 0.1 * torch.randn(D, device=DEV)
    full = conv1d_silu(xin, w, b)
    pre, cstate = conv1d_silu_state(xin[:, :L], w, b)
    assert rel(pre, full[:, :L]) <= 1e-6
    outs = []
    for t in range(T):
        o, cstate = conv1d_step(xin[:, L + t], cstate, w, b)
        outs.append(o)
    assert rel(torch.stack(outs, 1), full[:, L:]) <= 1e-6
    # the momentum scan: prefill with state_out, then single steps
    x = full
    delta = 0.5 * torch.randn(Bsz, L + T, D, device=DEV) - 2
    z = torch.randn(Bsz, L + T, D, device=DEV)
    A = -torch.arange(1, N + 1, device=DEV, dtype=torch.float32).repeat(D, 1)
    Bm = torch.randn(Bsz, L + T, N, device=DEV)
    Cm = torch.randn(Bsz, L + T, N, device=DEV)
    Dk = torch.randn(D, device=DEV)
    bias = 0.1 * torch.randn(D, device=DEV)
    kw = (0.7, 0.9)
    ref = ScanCall(x, delta, A, Bm, Cm, Dk, z, bias, True, *kw).forward(False)[0]
    _, _, st = ScanCall(x[:, :L].contiguous(), delta[:, :L].contiguous(), A, Bm[:, :L].contiguous(),
                        Cm[:, :L].contiguous(), Dk, z[:, :L].contiguous(), bias, True,
                        *kw).forward(False, want_state=True)
    h, v = st[:, :, 0].contiguous(), st[:, :, 1].contiguous()
    ys = []
    for t in range(T):
        y, h, v = mmscan_step(x[:, L + t], delta[:, L + t], A, Bm[:, L + t], Cm[:, L + t], h, v,
                              D=Dk, z=z[:, L + t], delta_bias=bias, delta_softplus=True,
                              beta=kw[0], alpha=kw[1])
        ys.append(y)
    assert rel(torch.stack(ys, 1), ref[:, L:]) <= TOL


def test_mmscan_step_vs_oracle():
    from momentummamba_b200.conv import mmscan_step
    g = torch.Generator().manual_seed(9)
    Bsz, D, N = 3, 200, 16
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    x, delta, z = r(Bsz, D), 0.5 * r(Bsz, D) - 2, r(Bsz, D)
    dbc = r(Bsz, 4 + 2 * N)                      # B, C as column slices of x_proj's output
    Bm, Cm = dbc[:, 4:4 + N], dbc[:, 4 + N:]
    A = -torch.arange(1, N + 1, dtype=torch.float64).repeat(D, 1)
    Dk, bias = r(D), 0.1 * r(D)
    h, v = r(Bsz, D, N), r(Bsz, D, N)
    yo, ho, vo = oc.mmscan_step(x, delta, A, Bm, Cm, h, v, Dk, z, bias, True, 0.8, 1.1)
    cu = lambda t: t.float().to(DEV)
    dbc_g = cu(dbc)
    hg, vg = cu(h), cu(v)
    y, h2, v2 = mmscan_step(cu(x), cu(delta), cu(A), dbc_g[:, 4:4 + N], dbc_g[:, 4 + N:], hg, vg,
                            D=cu(Dk), z=cu(z), delta_bias=cu(bias), delta_softplus=True, beta=0.8,
                            alpha=1.1, h_out=hg, v_out=vg)   # in place
    assert rel(y, yo) <= TOL and rel(hg, ho) <= TOL and rel(vg, vo) <= TOL
    # empty cache (the reference's h = v = None)
    yo, ho, vo = oc.mmscan_step(x, delta, A, Bm, Cm, None, None, Dk, None, bias, True, 0.8, 1.1)
    y, h2, v2 = mmscan_step(cu(x), cu(delta), cu(A), dbc_g[:, 4:4 + N], dbc_g[:, 4 + N:], None,
                            None, D=cu(Dk), delta_bias=cu(bias), delta_softplus=True, beta=0.8,
                            alpha=1.1)
    assert rel(y, yo) <= TOL and rel(h2, ho) <= TOL and rel(v2, vo) <= TOL


def _block(g):
    import momentummamba_b200.mamba_momentum as mm
    cfg = mm.MambaMomentumConfig(d_model=16, n_layers=1, d_state=16, expand_factor=2, d_conv=4,
                                 dt_rank=4, momentum_beta=0.8, momentum_alpha=0.9, bias=True,
                                 conv_bias=True)
    blk = mm.MambaMomentumBlock(cfg).to(DEV)
    blk.load_state_dict({k[2:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("p.")})
    return blk


def test_block_matches_reference_golden(golden_dir):
    torch.backends.cuda.matmul.allow_tf32 = False
    g = dict(np.load(os.path.join(golden_dir, "mm_block.npz")))
    blk = _block(g)
    x = torch.from_numpy(g["x"]).to(DEV).requires_grad_(True)
    y = blk(x)
    assert rel(y, g["y"]) <= TOL
    names = [k for k, _ in blk.named_parameters()]
    grads = torch.autograd.grad(y, [x] + [p for _, p in blk.named_parameters()],
                                torch.from_numpy(g["gy"]).to(DEV))
    assert rel(grads[0], g["dx"]) <= TOL
    for n, gr in zip(names, grads[1:]):
        assert rel(gr, g["g." + n]) <= TOL, n


def test_block_decode_matches_reference_golden(golden_dir):
    torch.backends.cuda.matmul.allow_tf32 = False
    g = dict(np.load(os.path.join(golden_dir, "mm_step.npz")))
    blk = _block(g)
    xs = torch.from_numpy(g["xs"]).to(DEV)
    cache = (None, None, torch.zeros(xs.shape[1], blk.config.d_inner, blk.config.d_conv - 1,
                                     device=DEV))
    ys = []
    with torch.no_grad():
        for t in range(xs.shape[0]):
            y, cache = blk.step(xs[t], cache)
            ys.append(y)
    assert rel(torch.stack(ys), g["ys"]) <= TOL
    for k, got in zip(("h", "v", "inputs"), cache):
        assert rel(got, g[k]) <= TOL, k
