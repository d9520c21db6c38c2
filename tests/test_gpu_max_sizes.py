"""The momentum scan at the largest single-GPU problem sizes of the benchmark
configurations, against the fp64 CPU oracle.

* Sequence classifier layer (B=256, T=300, D=512, N=16; softplus(delta + bias)
  and the SiLU(z) gate fused; fp32): outputs and every gradient against the
  oracle over the whole batch.
  Tolerance: max|gpu - ref| / max|ref| <= 1e-4.
* Long sequence (B=8, L=65536, D=2048, N=16; bf16 activations, fp32 state and
  sums; delta = softplus(0.5 N(0,1) - 2), A = -(n+1), D = 1, beta 0.9, no
  gate): the whole problem runs on the GPU.  Channels are independent, so the
  oracle checks a 16-channel slice of every sequence on the same bf16-rounded
  inputs: out, dx, ddelta, and the slice's dA, dD.
  Tolerances:
  - bf16 outputs (out, dx, ddelta): 4e-3, since bf16 rounding alone is up to
    2^-9 of the largest value;
  - fp32 sums (dA, dD): 2e-4, since each sums 524288 fp32 terms.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_classifier_layer_full_size():
    from test_gpu_mmscan import check_case, make_inputs
    rng = np.random.default_rng(11)
    inp = make_inputs(rng, 256, 300, 512, 16, z=True, bias=True)
    check_case(inp, softplus=True, beta=0.6, alpha=1.0)


def test_long_sequence_bf16_full_size():
    from momentummamba_b200 import selective_scan_momentum_fn
    Bsz, L, Dm, N = 8, 65536, 2048, 16
    beta, alpha = 0.9, 1.0
    g = torch.Generator(device=DEV).manual_seed(4)
    bf = torch.bfloat16
    x = torch.randn(Bsz, L, Dm, device=DEV, generator=g, dtype=bf).requires_grad_()
    delta = torch.empty(Bsz, L, Dm, device=DEV, dtype=bf)
    for b in range(Bsz):  # softplus(0.5 N(0,1) - 2), one sequence at a time (fp32 temporaries)
        r = torch.randn(L, Dm, device=DEV, generator=g)
        delta[b] = torch.nn.functional.softplus(0.5 * r - 2.0).to(bf)
    delta.requires_grad_()
    A = (-torch.arange(1, N + 1, device=DEV, dtype=torch.float32).repeat(Dm, 1)).requires_grad_()
    Bm = torch.randn(Bsz, L, N, device=DEV, generator=g, dtype=bf)
    Cm = torch.randn(Bsz, L, N, device=DEV, generator=g, dtype=bf)
    Dv = torch.ones(Dm, device=DEV).requires_grad_()
    dout = torch.randn(Bsz, L, Dm, device=DEV, generator=g, dtype=bf)

    y = selective_scan_momentum_fn(x, delta, A, Bm, Cm, Dv, beta=beta, alpha=alpha)
    gx, gd, gA, gD = torch.autograd.grad(y, [x, delta, A, Dv], dout)
    assert y.dtype == bf and gx.dtype == bf
    assert torch.isfinite(y).all() and torch.isfinite(gx).all() and torch.isfinite(gd).all()

    d0, dn = 1000, 16
    sl = slice(d0, d0 + dn)
    f64 = lambda t: t.detach().double().cpu().numpy()
    xo, do_, Bo, Co, go = (f64(t) for t in (x[:, :, sl], delta[:, :, sl], Bm, Cm,
                                             dout[:, :, sl]))
    Ao, Do = f64(A[sl]), f64(Dv[sl])
    yo = oracle.mmscan_fwd(xo, do_, Ao, Bo, Co, Do, None, None, False, beta, alpha)
    r = oracle.mmscan_bwd(xo, do_, Ao, Bo, Co, Do, None, None, False, beta, alpha, go)
    gxo, gdo, gAo, gDo = r[0], r[1], r[2], r[5]
    assert _rel(f64(y[:, :, sl]), yo) <= 4e-3
    assert _rel(f64(gx[:, :, sl]), gxo) <= 4e-3
    assert _rel(f64(gd[:, :, sl]), gdo) <= 4e-3
    assert _rel(f64(gA[sl]), gAo) <= 2e-4
    assert _rel(f64(gD[sl]), gDo) <= 2e-4
