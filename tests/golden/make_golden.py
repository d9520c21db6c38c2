"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run once, in a container that has the reference checkout (it is not needed
afterwards; the fixtures are committed):

    python tests/golden/make_golden.py /path/to/reference

Every fixture stores the seeded inputs, the upstream gradient it used, and the
reference's outputs and autograd gradients, all as float32 (complex64 for
complex tensors).  What each fixture exercises:

  mm_cfg0      MambaMomentumBlock.selective_scan_momentum, pscan_mode
               'pscan_sequential' (mamba_momentum.py:256-368 -> pscan.py), the
               B=2 L=256 D=64 N=16 beta=0.9 alpha=1 operator case
  mm_pad300    same, L=300 (PScan zero-pads to 512, pscan.py:176-182)
  mm_beta0     same, beta=0 (the single-pscan shortcut, mamba_momentum.py:343-347)
  mm_seq       _sequential_momentum_scan (mamba_momentum.py:415-435) on
               (B, L, ED, N) discretised tensors: the row-scan semantics of
               momentum_scan_cuda
  pscan_64     pscan(A, X) (pscan.py:160-234), L=64
  pscan_100    pscan(A, X), L=100 (padding path)
  lin_vec      mamba_linoss.parallel_scan_batched_complex (mamba_linoss.py:336-415)
  lin_pt       LinOSS_pytorch.parallel_scan_batched (LinOSS_pytorch.py:53-96), real F
  lin_im       LinOSS_pytorch.apply_linoss_im_complex (:153-195)
  lin_imex     LinOSS_pytorch.apply_linoss_imex_complex (:198-239)
  lin_layer_im / lin_layer_imex
               LinOSS_pytorch.LinOSSLayer forward on a (B, L, H) batch (vmap path)
  mlin_im / mlin_imex
               mamba_linoss.apply_linoss_vectorized(..., scan_algorithm='vectorized')
  mm_block     MambaMomentumBlock.forward (mamba_momentum.py:209-232: in_proj,
               causal depthwise conv1d + SiLU, x_proj, dt_proj + softplus, the
               momentum scan, SiLU(z) gate, out_proj) with its parameters,
               input, output, and the gradients of the input and every
               parameter for a random upstream gradient
  mm_step      the same block's step() (mamba_momentum.py:439-515) over 6
               tokens from an empty cache: the outputs and the final cache
  mm_state_dict.json
               parameter names and shapes of the reference MambaMomentum
               (d_model=128, n_layers=2, dt_rank=8): the module tree a drop-in
               must reproduce to load the reference's checkpoints
"""
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    t = t.detach()
    if t.is_complex():
        return t.to(torch.complex64).numpy()
    return t.to(torch.float32).numpy()


def _save(name, **arrs):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: (_np(v) if isinstance(v, torch.Tensor) else np.asarray(v))
                                 for k, v in arrs.items()})
    print("wrote", path, os.path.getsize(path), "bytes")


def mm_inputs(g, Bsz, L, Dm, N):
    """Operator-case distributions: x~N(0,1); delta=softplus(0.5*N(0,1)-2);
    A[d,n]=-(n+1); B,C~N(0,1); D=1."""
    x = torch.randn(Bsz, L, Dm, generator=g)
    delta = F.softplus(0.5 * torch.randn(Bsz, L, Dm, generator=g) - 2.0)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(Dm, 1)
    Bm = torch.randn(Bsz, L, N, generator=g)
    Cm = torch.randn(Bsz, L, N, generator=g)
    D = torch.ones(Dm)
    return x, delta, A, Bm, Cm, D


def gen_mm(ref, name, Bsz, L, Dm, N, beta, alpha, seed):
    mm = ref["mamba_momentum"]
    g = torch.Generator().manual_seed(seed)
    x, delta, A, Bm, Cm, D = mm_inputs(g, Bsz, L, Dm, N)
    cfg = mm.MambaMomentumConfig(d_model=Dm // 2, n_layers=1, d_state=N, expand_factor=2,
                                 momentum_beta=beta, momentum_alpha=alpha,
                                 pscan_mode="pscan_sequential")
    blk = mm.MambaMomentumBlock(cfg)
    ins = [t.clone().requires_grad_(True) for t in (x, delta, A, Bm, Cm, D)]
    y = blk.selective_scan_momentum(*ins)
    gy = torch.randn(y.shape, generator=g)
    grads = torch.autograd.grad(y, ins, gy)
    _save(name, x=x, delta=delta, A=A, B=Bm, C=Cm, D=D, beta=beta, alpha=alpha, y=y, gy=gy,
          dx=grads[0], ddelta=grads[1], dA=grads[2], dB=grads[3], dC=grads[4], dD=grads[5])


def gen_mm_seq(ref, seed):
    mm = ref["mamba_momentum"]
    g = torch.Generator().manual_seed(seed)
    Bsz, L, ED, N = 2, 96, 8, 4
    beta = 0.75
    dA = torch.exp(-torch.rand(Bsz, L, ED, N, generator=g) * 0.5)
    u = torch.randn(Bsz, L, ED, N, generator=g)
    cfg = mm.MambaMomentumConfig(d_model=4, n_layers=1, d_state=N, momentum_beta=beta)
    blk = mm.MambaMomentumBlock(cfg)
    a_, u_ = dA.clone().requires_grad_(True), u.clone().requires_grad_(True)
    h = blk._sequential_momentum_scan(a_, beta, u_)
    gh = torch.randn(h.shape, generator=g)
    ga, gu = torch.autograd.grad(h, [a_, u_], gh)
    _save("mm_seq", deltaA=dA, u=u, beta=beta, h=h, gh=gh, ddeltaA=ga, du=gu)


def _mm_block(ref, seed):
    mm = ref["mamba_momentum"]
    torch.manual_seed(seed)
    cfg = mm.MambaMomentumConfig(d_model=16, n_layers=1, d_state=16, expand_factor=2,
                                 d_conv=4, dt_rank=4, momentum_beta=0.8, momentum_alpha=0.9,
                                 bias=True, conv_bias=True)
    blk = mm.MambaMomentumBlock(cfg)
    with torch.no_grad():   # move A_log, D, conv bias off their constant inits
        blk.A_log.add_(0.1 * torch.randn(blk.A_log.shape))
        blk.D.add_(0.2 * torch.randn(blk.D.shape))
        blk.conv1d.bias.add_(0.1 * torch.randn(blk.conv1d.bias.shape))
    params = {k: v.detach().clone() for k, v in blk.state_dict().items()}
    return blk, params


def gen_mm_block(ref, seed):
    blk, params = _mm_block(ref, seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, 37, 16, generator=g)
    xi = x.clone().requires_grad_(True)
    y = blk(xi)
    gy = torch.randn(y.shape, generator=g)
    names = [k for k, _ in blk.named_parameters()]
    grads = torch.autograd.grad(y, [xi] + [p for _, p in blk.named_parameters()], gy)
    _save("mm_block", x=x, y=y, gy=gy, dx=grads[0],
          **{"p." + k: v for k, v in params.items()},
          **{"g." + k: gr for k, gr in zip(names, grads[1:])})


def gen_mm_step(ref, seed):
    blk, params = _mm_block(ref, seed)
    g = torch.Generator().manual_seed(seed + 100)
    Bsz, T = 3, 6
    ed, n, w = blk.config.d_inner, blk.config.d_state, blk.config.d_conv
    xs = torch.randn(T, Bsz, 16, generator=g)
    cache = (None, None, torch.zeros(Bsz, ed, w - 1))
    ys = []
    with torch.no_grad():
        for t in range(T):
            y, cache = blk.step(xs[t], cache)
            ys.append(y)
    h, v, inputs = cache
    _save("mm_step", xs=xs, ys=torch.stack(ys), h=h, v=v, inputs=inputs,
          **{"p." + k: val for k, val in params.items()})


def gen_pscan(ref, name, L, seed):
    pscan = ref["pscan"].pscan
    g = torch.Generator().manual_seed(seed)
    Bsz, Dm, N = 2, 6, 4
    A = torch.exp(-torch.rand(Bsz, L, Dm, N, generator=g))
    X = torch.randn(Bsz, L, Dm, N, generator=g)
    a_, x_ = A.clone().requires_grad_(True), X.clone().requires_grad_(True)
    H = pscan(a_, x_)
    gH = torch.randn(H.shape, generator=g)
    gA, gX = torch.autograd.grad(H, [a_, x_], gH)
    _save(name, A=A, X=X, H=H, gH=gH, dA=gA, dX=gX)


def lin_M(g, Bsz, L, P):
    """Random IM-like transitions: stable 2x2 blocks per (b, l, p)."""
    dt = torch.rand(Bsz, L, P, generator=g) * 0.5 + 0.05
    A = torch.rand(Bsz, L, P, generator=g)
    S = 1.0 / (1.0 + dt * dt * A)
    return torch.cat([1.0 - dt * dt * A * S, -dt * A * S, dt * S, S], dim=-1)


def gen_lin_vec(ref, seed):
    ml = ref["mamba_linoss"]
    g = torch.Generator().manual_seed(seed)
    Bsz, L, P = 2, 100, 8
    M = lin_M(g, Bsz, L, P)
    Fc = torch.complex(torch.randn(Bsz, L, 2 * P, generator=g), torch.randn(Bsz, L, 2 * P, generator=g))
    M_, F_ = M.clone().requires_grad_(True), Fc.clone().requires_grad_(True)
    Ms, X = ml.parallel_scan_batched_complex(M_, F_)
    gX = torch.complex(torch.randn(X.shape, generator=g), torch.randn(X.shape, generator=g))
    gMs = torch.randn(Ms.shape, generator=g) * 0.1
    loss = (X.real * gX.real + X.imag * gX.imag).sum() + (Ms * gMs).sum()
    dM, dF = torch.autograd.grad(loss, [M_, F_])
    _save("lin_vec", M=M, F=Fc, Mscan=Ms, X=X, gX=gX, gMscan=gMs, dM=dM, dF=dF)


def gen_lin_pt(ref, seed):
    lp = ref["LinOSS_pytorch"]
    g = torch.Generator().manual_seed(seed)
    L, P = 77, 6
    M = lin_M(g, 1, L, P)[0]
    Fr = torch.randn(L, 2 * P, generator=g)
    M_, F_ = M.clone().requires_grad_(True), Fr.clone().requires_grad_(True)
    Ms, X = lp.parallel_scan_batched(M_, F_)
    gX = torch.randn(X.shape, generator=g)
    dM, dF = torch.autograd.grad(X, [M_, F_], gX)
    _save("lin_pt", M=M, F=Fr, Mscan=Ms, X=X, gX=gX, dM=dM, dF=dF)


def linoss_params(g, P, H):
    A_diag = torch.rand(P, generator=g)
    Br = torch.randn(P, H, generator=g) / math.sqrt(H)
    Bi = torch.randn(P, H, generator=g) / math.sqrt(H)
    Cr = torch.randn(H, P, generator=g) / math.sqrt(H)
    Ci = torch.randn(H, P, generator=g) / math.sqrt(H)
    lo, hi = math.log(1e-3), math.log(1e-1)
    step = torch.exp(lo + (hi - lo) * torch.rand(P, generator=g))
    return A_diag, Br, Bi, Cr, Ci, step


def gen_lin_apply(ref, disc, seed):
    lp = ref["LinOSS_pytorch"]
    g = torch.Generator().manual_seed(seed)
    L, H, P = 64, 16, 8
    A_diag, Br, Bi, Cr, Ci, step = linoss_params(g, P, H)
    u = torch.randn(L, H, generator=g)
    ins = [t.clone().requires_grad_(True) for t in (A_diag, Br, Bi, Cr, Ci, u, step)]
    fn = lp.apply_linoss_im_complex if disc == "IM" else lp.apply_linoss_imex_complex
    y = fn(*ins)
    gy = torch.randn(y.shape, generator=g)
    gr = torch.autograd.grad(y, ins, gy)
    _save("lin_" + disc.lower(), A_diag=A_diag, B_real=Br, B_imag=Bi, C_real=Cr, C_imag=Ci,
          u=u, step=step, y=y, gy=gy, dA_diag=gr[0], dB_real=gr[1], dB_imag=gr[2],
          dC_real=gr[3], dC_imag=gr[4], du=gr[5], dstep=gr[6])


def gen_lin_layer(ref, disc, seed):
    lp = ref["LinOSS_pytorch"]
    torch.manual_seed(seed)
    Bsz, L, H, P = 2, 48, 16, 8
    layer = lp.LinOSSLayer(P, H, disc)
    g = torch.Generator().manual_seed(seed + 1)
    u = torch.randn(Bsz, L, H, generator=g)
    u_ = u.clone().requires_grad_(True)
    y = layer(u_)
    gy = torch.randn(y.shape, generator=g)
    params = [layer.A_diag, layer.B_real, layer.B_imag, layer.C_real, layer.C_imag, layer.D,
              layer.steps]
    gr = torch.autograd.grad(y, [u_] + params, gy)
    _save("lin_layer_" + disc.lower(), u=u, A_diag=layer.A_diag, B_real=layer.B_real,
          B_imag=layer.B_imag, C_real=layer.C_real, C_imag=layer.C_imag, D=layer.D,
          steps=layer.steps, y=y, gy=gy, du=gr[0], dA_diag=gr[1], dB_real=gr[2],
          dB_imag=gr[3], dC_real=gr[4], dC_imag=gr[5], dD=gr[6], dsteps=gr[7])


def gen_mlin(ref, disc, seed):
    ml = ref["mamba_linoss"]
    g = torch.Generator().manual_seed(seed)
    Bsz, L, ED, P = 2, 40, 12, 8
    A_diag = torch.exp(torch.rand(P, generator=g) * 2.0)
    Br, Bi, Cr, Ci = (torch.randn(Bsz, L, P, generator=g) * 0.5 for _ in range(4))
    x = torch.randn(Bsz, L, ED, generator=g)
    delta = F.softplus(torch.randn(Bsz, L, ED, generator=g) * 0.5 - 2.0)
    ins = [t.clone().requires_grad_(True) for t in (A_diag, Br, Bi, Cr, Ci, x, delta)]
    y = ml.apply_linoss_vectorized(disc, ins[0], ins[1], ins[2], ins[3], ins[4], ins[5], ins[6],
                                   scan_algorithm="vectorized")
    gy = torch.randn(y.shape, generator=g)
    gr = torch.autograd.grad(y, ins, gy, allow_unused=True)
    dx = gr[5] if gr[5] is not None else torch.zeros_like(x)
    _save("mlin_" + disc.lower(), A_diag=A_diag, B_real=Br, B_imag=Bi, C_real=Cr, C_imag=Ci,
          x=x, delta=delta, y=y, gy=gy, dA_diag=gr[0], dB_real=gr[1], dB_imag=gr[2],
          dC_real=gr[3], dC_imag=gr[4], dx=dx, ddelta=gr[6])


def gen_state_dict(ref):
    import json
    mm = ref["mamba_momentum"]
    m = mm.MambaMomentum(mm.MambaMomentumConfig(d_model=128, n_layers=2, dt_rank=8))
    keys = {k: list(v.shape) for k, v in m.state_dict().items()}
    path = os.path.join(HERE, "mm_state_dict.json")
    with open(path, "w") as f:
        json.dump(keys, f, indent=0, sort_keys=True)
    print("wrote", path)


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference source directory>")
    refdir = sys.argv[1]
    sys.path.insert(0, refdir)
    import importlib
    ref = {m: importlib.import_module(m)
           for m in ("pscan", "mamba_momentum", "mamba_linoss", "LinOSS_pytorch")}
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gen_mm(ref, "mm_cfg0", 2, 256, 64, 16, 0.9, 1.0, seed=0)
    gen_mm(ref, "mm_pad300", 1, 300, 16, 8, 0.6, 0.5, seed=1)
    gen_mm(ref, "mm_beta0", 2, 64, 16, 16, 0.0, 1.0, seed=2)
    gen_mm_seq(ref, seed=3)
    gen_pscan(ref, "pscan_64", 64, seed=4)
    gen_pscan(ref, "pscan_100", 100, seed=5)
    gen_lin_vec(ref, seed=6)
    gen_lin_pt(ref, seed=7)
    gen_lin_apply(ref, "IM", seed=8)
    gen_lin_apply(ref, "IMEX", seed=9)
    gen_lin_layer(ref, "IM", seed=10)
    gen_lin_layer(ref, "IMEX", seed=11)
    gen_mlin(ref, "IM", seed=12)
    gen_mlin(ref, "IMEX", seed=13)
    gen_mm_block(ref, seed=14)
    gen_mm_step(ref, seed=14)
    gen_state_dict(ref)


if __name__ == "__main__":
    main()
