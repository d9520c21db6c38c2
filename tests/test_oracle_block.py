"""The momentum block's host logic (momentummamba_b200/mamba_momentum.py) with
the oracle's fp64 restatements in place of the CUDA ops, against the
reference's own block forward/backward and decode steps (tests/golden/mm_block,
mm_step).  Pins the restatements of the conv producer and the decode step that
the GPU tests compare the kernels with."""
import os

import numpy as np
import pytest
import torch

from oracle import composite as oc

TOL = 2e-5   # fp32 reference vs fp64 restatement


def _patch(monkeypatch):
    import momentummamba_b200.mamba_momentum as mm

    def scan(x, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False, beta=0.6,
             alpha=1.0):
        return oc.mmscan(x, delta, A, B, C, D, z, delta_bias, delta_softplus, beta, alpha)

    monkeypatch.setattr(mm, "selective_scan_momentum_fn", scan)
    monkeypatch.setattr(mm, "conv1d_silu", oc.conv1d_silu)
    monkeypatch.setattr(mm, "conv1d_step", oc.conv1d_step)
    monkeypatch.setattr(mm, "mmscan_step", oc.mmscan_step)
    return mm


def _block(mm, g):
    cfg = mm.MambaMomentumConfig(d_model=16, n_layers=1, d_state=16, expand_factor=2, d_conv=4,
                                 dt_rank=4, momentum_beta=0.8, momentum_alpha=0.9, bias=True,
                                 conv_bias=True)
    blk = mm.MambaMomentumBlock(cfg).double()
    blk.load_state_dict({k[2:]: torch.from_numpy(v).double() for k, v in g.items()
                         if k.startswith("p.")})
    return blk


def rel(a, b):
    a = a.detach().numpy() if isinstance(a, torch.Tensor) else a
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_block_forward_backward_matches_reference(golden_dir, monkeypatch):
    mm = _patch(monkeypatch)
    g = dict(np.load(os.path.join(golden_dir, "mm_block.npz")))
    blk = _block(mm, g)
    x = torch.from_numpy(g["x"]).double().requires_grad_(True)
    y = blk(x)
    assert rel(y, g["y"]) < TOL
    names = [k for k, _ in blk.named_parameters()]
    grads = torch.autograd.grad(y, [x] + [p for _, p in blk.named_parameters()],
                                torch.from_numpy(g["gy"]).double())
    assert rel(grads[0], g["dx"]) < TOL
    for n, gr in zip(names, grads[1:]):
        assert rel(gr, g["g." + n]) < TOL, n


def test_block_decode_steps_match_reference(golden_dir, monkeypatch):
    mm = _patch(monkeypatch)
    g = dict(np.load(os.path.join(golden_dir, "mm_step.npz")))
    blk = _block(mm, g)
    xs = torch.from_numpy(g["xs"]).double()
    Bsz, ed = xs.shape[1], blk.config.d_inner
    cache = (None, None, torch.zeros(Bsz, ed, blk.config.d_conv - 1, dtype=torch.float64))
    ys = []
    with torch.no_grad():
        for t in range(xs.shape[0]):
            y, cache = blk.step(xs[t], cache)
            ys.append(y)
    assert rel(torch.stack(ys), g["ys"]) < TOL
    for k, got in zip(("h", "v", "inputs"), cache):
        assert rel(got, g[k]) < TOL, k
