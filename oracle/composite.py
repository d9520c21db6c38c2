"""Autograd wrappers around the C oracle, plus fp64 restatements of the reference
glue that surrounds the scans (discretisation of LinOSS, output contraction).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Everything here runs on
the CPU in float64 unless ``prec='f32'`` is asked for.  The scan cores are the
C restatements; the glue is ordinary torch CPU arithmetic restating the cited
reference lines, differentiated by autograd.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import mmscan_bwd, mmscan_fwd, rows_bwd, rows_fwd, scan2_bwd, scan2_fwd

_F64 = torch.float64


def _t(a, like):
    return torch.from_numpy(np.ascontiguousarray(a)).to(like.dtype if not np.iscomplexobj(a)
                                                          else torch.complex128)


def _n(t):
    return None if t is None else t.detach().cpu().numpy()


class MMScanFn(torch.autograd.Function):
    """Momentum selective scan (mamba_momentum.py:256-323, gate :227-229)."""

    @staticmethod
    def forward(ctx, x, delta, A, B, C, D, z, delta_bias, softplus, beta, alpha, prec):
        out = mmscan_fwd(_n(x), _n(delta), _n(A), _n(B), _n(C), _n(D), _n(z), _n(delta_bias),
                         softplus, beta, alpha, prec=prec)
        ctx.save_for_backward(x, delta, A, B, C, D, z, delta_bias)
        ctx.cfg = (softplus, beta, alpha, prec)
        return _t(out, x)

    @staticmethod
    def backward(ctx, g):
        x, delta, A, B, C, D, z, delta_bias = ctx.saved_tensors
        softplus, beta, alpha, prec = ctx.cfg
        r = mmscan_bwd(_n(x), _n(delta), _n(A), _n(B), _n(C), _n(D), _n(z), _n(delta_bias),
                       softplus, beta, alpha, _n(g), prec=prec)
        conv = [None if a is None else _t(a, x) for a in r]
        dx, ddelta, dA, dB, dC, dD, dz, ddb = conv
        return dx, ddelta, dA, dB, dC, dD, dz, ddb, None, None, None, None


def mmscan(x, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
           beta=0.6, alpha=1.0, prec="f64"):
    return MMScanFn.apply(x, delta, A, B, C, D, z, delta_bias, delta_softplus, beta, alpha, prec)


class RowsFn(torch.autograd.Function):
    """Row scan v = beta*v + u ; h = a*h + v (momentum_scan_cuda.py:22-87)."""

    @staticmethod
    def forward(ctx, a, beta, u, prec):
        h = rows_fwd(_n(a), beta, _n(u), prec=prec)
        h = _t(h, a)
        ctx.save_for_backward(a, h)
        ctx.cfg = (beta, prec)
        return h

    @staticmethod
    def backward(ctx, g):
        a, h = ctx.saved_tensors
        beta, prec = ctx.cfg
        da, du = rows_bwd(_n(g), _n(a), beta, _n(h), prec=prec)
        return _t(da, a), None, _t(du, a), None


def rows(a, beta, u, prec="f64"):
    return RowsFn.apply(a, beta, u, prec)


def pscan(A, X, prec="f64"):
    """PScan semantics (pscan.py:160-234) through the row scan with beta = 0."""
    Bsz, L = A.shape[0], A.shape[1]
    shp = A.shape
    a = A.reshape(Bsz, L, -1).transpose(1, 2).reshape(-1, L)
    x = X.reshape(Bsz, L, -1).transpose(1, 2).reshape(-1, L)
    h = rows(a, 0.0, x, prec)
    return h.reshape(Bsz, -1, L).transpose(1, 2).reshape(shp)


class Scan2Fn(torch.autograd.Function):
    """2x2 scan x_t = M_t x_{t-1} + F_t (mamba_linoss.py:336-415, :561-605)."""

    @staticmethod
    def forward(ctx, M, Fv, prec):
        Ms, X = scan2_fwd(_n(M), _n(Fv), prec=prec, return_mscan=True)
        Ms = _t(Ms, M)
        X = torch.from_numpy(np.ascontiguousarray(X)).to(Fv.dtype)
        ctx.save_for_backward(M, Ms, X)
        ctx.prec = prec
        return Ms, X

    @staticmethod
    def backward(ctx, gMs, gX):
        M, Ms, X = ctx.saved_tensors
        dM, dF = scan2_bwd(_n(M), _n(X), _n(gX), Mscan=_n(Ms), gMscan=_n(gMs), prec=ctx.prec)
        dM = _t(dM, M)
        dF = torch.from_numpy(np.ascontiguousarray(dF)).to(X.dtype)
        return dM, dF, None


def scan2(M, Fv, prec="f64"):
    return Scan2Fn.apply(M, Fv, prec)


# ---------------------------------------------------------------------------
# LinOSS layer glue (LinOSS_pytorch.py:135-239, :258-312)
# ---------------------------------------------------------------------------
def _linoss_matrices(disc, A_diag, step):
    if disc == "IM":
        # LinOSS_pytorch.py:164-168
        S = 1.0 / (1.0 + step ** 2 * A_diag)
        m11 = 1.0 - step ** 2 * A_diag * S
        m12 = -step * A_diag * S
        m21 = step * S
        m22 = S
        f1 = m11 * step
        f2 = m21 * step
    elif disc == "IMEX":
        # LinOSS_pytorch.py:209-222
        m11 = torch.ones_like(A_diag)
        m12 = -step * A_diag
        m21 = step * torch.ones_like(A_diag)
        m22 = 1.0 - step ** 2 * A_diag
        f1 = step
        f2 = step ** 2
    else:
        raise ValueError(disc)
    return torch.cat([m11, m12, m21, m22]), f1, f2


def linoss_apply(disc, A_diag, B_real, B_imag, C_real, C_imag, u, step, prec="f64"):
    """apply_linoss_im_complex / apply_linoss_imex_complex for u of shape (L, H)
    or (Bsz, L, H): Bu = B u (complex), time-invariant M, scan, y = Re(C x2)."""
    squeeze = u.dim() == 2
    if squeeze:
        u = u.unsqueeze(0)
    Bsz, L, H = u.shape
    P = A_diag.shape[0]
    Bu_r = torch.einsum("ph,blh->blp", B_real, u)
    Bu_i = torch.einsum("ph,blh->blp", B_imag, u)
    Mv, f1, f2 = _linoss_matrices(disc, A_diag, step)
    M = Mv.reshape(1, 1, 4 * P).expand(Bsz, L, 4 * P)
    Fv = torch.complex(torch.cat([f1 * Bu_r, f2 * Bu_r], -1), torch.cat([f1 * Bu_i, f2 * Bu_i], -1))
    _, X = scan2(M, Fv, prec)
    x2 = X[..., P:]
    y = torch.einsum("hp,blp->blh", C_real, x2.real) - torch.einsum("hp,blp->blh", C_imag, x2.imag)
    return y[0] if squeeze else y


def linoss_layer(disc, u, A_diag, B_real, B_imag, C_real, C_imag, D, steps, prec="f64"):
    """LinOSSLayer.forward (LinOSS_pytorch.py:258-312): relu(A), sigmoid(steps), + D*u."""
    A = F.relu(A_diag)
    step = torch.sigmoid(steps)
    y = linoss_apply(disc, A, B_real, B_imag, C_real, C_imag, u, step, prec)
    return y + u * D


def mlinoss_apply(disc, A_diag, B_real, B_imag, C_real, C_imag, x, delta, prec="f64"):
    """apply_linoss_vectorized (mamba_linoss.py:608-677) with a correct scan."""
    Bsz, L, ED = x.shape
    P = A_diag.shape[0]
    Bc = torch.complex(B_real, B_imag)
    Cc = torch.complex(C_real, C_imag)
    dbar = delta.mean(dim=-1, keepdim=True)                  # :622
    Bu = Bc * dbar                                           # :626
    Ad = A_diag.reshape(1, 1, P)
    if disc == "IM":                                         # :630-642
        S = 1.0 / (1.0 + dbar ** 2 * Ad)
        m11 = 1.0 - dbar ** 2 * Ad * S
        m12 = -dbar * Ad * S
        m21 = dbar * S
        m22 = S
        Fv = torch.cat([m11 * Bu, m21 * Bu], dim=-1)
    elif disc == "IMEX":                                     # :646-657
        m11 = torch.ones(Bsz, L, P, dtype=delta.dtype)
        m12 = -dbar * Ad
        m21 = dbar * torch.ones(Bsz, L, P, dtype=delta.dtype)
        m22 = 1.0 - dbar ** 2 * Ad
        Fv = torch.cat([Bu, Bu * dbar], dim=-1)
    else:
        raise ValueError(disc)
    M = torch.cat([m11, m12, m21, m22], dim=-1)
    _, X = scan2(M, Fv, prec)
    y = torch.sum(Cc * X[..., P:], dim=-1).real              # :668-672
    return y.unsqueeze(-1).expand(-1, -1, ED)                # :675


def to64(*ts):
    out = []
    for t in ts:
        if t is None:
            out.append(None)
            continue
        t = torch.as_tensor(t)
        t = t.to(torch.complex128) if t.is_complex() else t.to(_F64)
        out.append(t.detach().clone().requires_grad_(True))
    return out


# ---------------------------------------------------------------------------
# the momentum block's producer and decode step, fp64 torch restatements
# ---------------------------------------------------------------------------
def conv1d_silu(x, weight, bias=None, state_in=None):
    """silu(causal depthwise conv1d over time) of x (B, L, D)
    (mamba_momentum.py:217-223: conv1d with groups = D, padding = W-1, first L
    outputs); state_in (B, D, W-1) are the inputs before t = 0."""
    Bsz, L, D = x.shape
    W = weight.shape[-1]
    xt = x.transpose(1, 2)
    if state_in is not None:
        y = F.conv1d(torch.cat([state_in, xt], 2), weight.reshape(D, 1, W), bias, groups=D)
    else:
        y = F.conv1d(xt, weight.reshape(D, 1, W), bias, padding=W - 1, groups=D)[:, :, :L]
    return F.silu(y.transpose(1, 2))


def conv1d_step(x, conv_state, weight, bias=None, out_state=None):
    """One token (mamba_momentum.py:455-459, :466): (silu(conv over
    [conv_state | x]), the shifted state)."""
    D, W = x.shape[1], weight.shape[-1]
    cat = torch.cat([conv_state, x.unsqueeze(2)], 2)
    y = F.conv1d(cat, weight.reshape(D, 1, W), bias, padding=W - 1, groups=D)[:, :, W - 1]
    return F.silu(y), cat[:, :, 1:]


def mmscan_step(x, delta, A, B, C, h=None, v=None, D=None, z=None, delta_bias=None,
                delta_softplus=False, beta=0.6, alpha=1.0, h_out=None, v_out=None):
    """One token of the momentum scan (mamba_momentum.py:473-515) and the block's
    gate (:461-464): (y, h, v)."""
    dt = delta if delta_bias is None else delta + delta_bias
    if delta_softplus:
        dt = F.softplus(dt)
    a = torch.exp(dt.unsqueeze(-1) * A)
    u = alpha * (dt.unsqueeze(-1) * B.unsqueeze(1)) * x.unsqueeze(-1)
    if h is None:
        h = torch.zeros_like(u)
    if v is None:
        v = torch.zeros_like(u)
    v = beta * v + u
    h = a * h + v
    y = (h * C.unsqueeze(1)).sum(-1)
    if D is not None:
        y = y + D * x
    if z is not None:
        y = y * F.silu(z)
    return y, h, v
