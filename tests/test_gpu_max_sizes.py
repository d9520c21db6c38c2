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
  inputs: out, dx, ddelta, and the slice's dA, dD.  Sequences are independent
  too, so the oracle also runs the whole first sequence (all 2048 channels, all
  65536 steps): out, dx, ddelta and that sequence's dB, dC, which sum over every
  channel and so cannot be checked on a channel slice.
  Tolerances:
  - bf16 outputs (out, dx, ddelta) and the gradients of the bf16 inputs B and
    C (summed in fp32 over the 2048 channels, then returned in their input's
    dtype, bf16): 4e-3, since bf16 rounding alone is up to 2^-9 of the largest
    value (2^-8 relative spacing, halved by rounding to nearest), with room for
    the fp32 arithmetic before the rounding;
  - fp32 sums (dA, dD over 524288 terms each): 2e-4.
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
    Bm = torch.randn(Bsz, L, N, device=DEV, generator=g, dtype=bf).requires_grad_()
    Cm = torch.randn(Bsz, L, N, device=DEV, generator=g, dtype=bf).requires_grad_()
    Dv = torch.ones(Dm, device=DEV).requires_grad_()
    dout = torch.randn(Bsz, L, Dm, device=DEV, generator=g, dtype=bf)

    y = selective_scan_momentum_fn(x, delta, A, Bm, Cm, Dv, beta=beta, alpha=alpha)
    gx, gd, gA, gB, gC, gD = torch.autograd.grad(y, [x, delta, A, Bm, Cm, Dv], dout)
    assert y.dtype == bf and gx.dtype == bf
    assert torch.isfinite(y).all() and torch.isfinite(gx).all() and torch.isfinite(gd).all()
    assert torch.isfinite(gB).all() and torch.isfinite(gC).all()

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
    del xo, do_, go, yo, r

    # the whole first sequence (every channel): its dB and dC sum over all of them
    xo, do_, Bo, Co, go = (f64(t[:1]) for t in (x, delta, Bm, Cm, dout))
    yo = oracle.mmscan_fwd(xo, do_, f64(A), Bo, Co, f64(Dv), None, None, False, beta, alpha)
    r = oracle.mmscan_bwd(xo, do_, f64(A), Bo, Co, f64(Dv), None, None, False, beta, alpha, go)
    assert _rel(f64(y[:1]), yo) <= 4e-3
    assert _rel(f64(gx[:1]), r[0]) <= 4e-3
    assert _rel(f64(gd[:1]), r[1]) <= 4e-3
    assert gB.dtype == bf and gC.dtype == bf
    assert _rel(f64(gB[:1]), r[3]) <= 4e-3
    assert _rel(f64(gC[:1]), r[4]) <= 4e-3
