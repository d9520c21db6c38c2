"""Fused momentum selective scan (forward + backward) on the sm_100a kernels.

``selective_scan_momentum_fn`` is the functional form of
``MambaMomentumBlock.selective_scan_momentum`` (mamba_momentum.py:256-323):

    dt  = softplus(delta + delta_bias) if delta_softplus else delta
    a   = exp(dt * A);  u = alpha * dt * B * x
    v_t = beta * v_{t-1} + u_t ;  h_t = a_t * h_{t-1} + v_t
    y   = sum_n C * h + D * x ;   out = y * silu(z) if z is given

with the block's softplus (mamba_momentum.py:247) and SiLU gate (:227-229)
optionally fused.  The forward keeps (h, v) every 8 steps for the backward,
which recomputes the states from there; nothing of size B*L*D*N is ever
materialised.  Gradients: x, delta, A, B, C, D, z, delta_bias (beta and alpha
are Python floats without gradient, as in momentum_scan_cuda.py:251).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_SUPPORTED_N = (8, 16, 32, 64)


def _padded_state(N: int) -> int:
    for n in _SUPPORTED_N:
        if N <= n:
            return n
    raise RuntimeError(f"momentummamba_b200: d_state={N} > 64 is not supported")


def _prep(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """fp32 with a unit-stride last dimension (any other strides are passed on)."""
    if t is None:
        return None
    if t.dtype != torch.float32:
        t = t.float()
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def _pad_last(t: torch.Tensor, n: int) -> torch.Tensor:
    if t.shape[-1] == n:
        return t
    out = t.new_zeros(*t.shape[:-1], n)
    out[..., : t.shape[-1]] = t
    return out


def _strides(t: Optional[torch.Tensor]):
    if t is None:
        return (0, 0)
    return (t.stride(0), t.stride(1))


def _desc(x, delta, z, B, C, N, beta, alpha, softplus):
    d = _lib.MMScanDesc()
    d.batch, d.seqlen, d.dim = x.shape
    d.dstate = N
    d.x_stride[:] = _strides(x)
    d.delta_stride[:] = _strides(delta)
    d.z_stride[:] = _strides(z)
    d.B_stride[:] = _strides(B)
    d.C_stride[:] = _strides(C)
    d.beta = float(beta)
    d.alpha = float(alpha)
    d.delta_softplus = 1 if softplus else 0
    return d


class SelectiveScanMomentumFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, delta, A, B, C, D, z, delta_bias, delta_softplus, beta, alpha):
        _lib.require_cuda(x, delta, A, B, C, D, z, delta_bias)
        lib = _lib.load()
        N0 = A.shape[1]
        N = _padded_state(N0)
        x, delta, z = _prep(x), _prep(delta), _prep(z)
        A, B, C = _prep(A).contiguous(), _prep(B), _prep(C)
        D = None if D is None else _prep(D).contiguous()
        delta_bias = None if delta_bias is None else _prep(delta_bias).contiguous()
        if N != N0:
            A, B, C = _pad_last(A, N), _pad_last(B, N), _pad_last(C, N)
        Bsz, L, Dm = x.shape
        if delta.shape != x.shape or (z is not None and z.shape != x.shape):
            raise ValueError("x, delta and z must share the shape (batch, seqlen, dim)")
        if A.shape[0] != Dm or B.shape != (Bsz, L, N) or C.shape != (Bsz, L, N):
            raise ValueError("A must be (dim, d_state); B and C (batch, seqlen, d_state)")
        out = torch.empty((Bsz, L, Dm), device=x.device, dtype=torch.float32)
        need_grad = any(ctx.needs_input_grad[:8])
        ckpt = None
        if need_grad:
            n = lib.mmb_mmscan_ckpt_floats(Bsz, L, Dm, N)
            ckpt = torch.empty(n, device=x.device, dtype=torch.float32)
        desc = _desc(x, delta, z, B, C, N, beta, alpha, delta_softplus)
        with torch.cuda.device(x.device):
            st = lib.mmb_mmscan_fwd(desc, _lib.ptr(x), _lib.ptr(delta), _lib.ptr(A), _lib.ptr(B),
                                    _lib.ptr(C), _lib.ptr(D), _lib.ptr(z), _lib.ptr(delta_bias),
                                    _lib.ptr(out), _lib.ptr(ckpt), _lib.stream_of(x))
        _lib.check(st, "mmb_mmscan_fwd")
        ctx.save_for_backward(x, delta, A, B, C, D, z, delta_bias, ckpt)
        ctx.cfg = (N0, N, bool(delta_softplus), float(beta), float(alpha))
        return out

    @staticmethod
    def backward(ctx, dout):
        lib = _lib.load()
        x, delta, A, B, C, D, z, delta_bias, ckpt = ctx.saved_tensors
        N0, N, softplus, beta, alpha = ctx.cfg
        dout = dout.float().contiguous()
        Bsz, L, Dm = x.shape
        dev = x.device
        f32 = torch.float32
        dx = torch.empty((Bsz, L, Dm), device=dev, dtype=f32)
        ddelta = torch.empty((Bsz, L, Dm), device=dev, dtype=f32)
        dA = torch.empty((Dm, N), device=dev, dtype=f32)
        dB = torch.empty((Bsz, L, N), device=dev, dtype=f32)
        dC = torch.empty((Bsz, L, N), device=dev, dtype=f32)
        dD = torch.empty((Dm,), device=dev, dtype=f32) if D is not None else None
        dz = torch.empty((Bsz, L, Dm), device=dev, dtype=f32) if z is not None else None
        ddb = torch.empty((Dm,), device=dev, dtype=f32) if delta_bias is not None else None
        desc = _desc(x, delta, z, B, C, N, beta, alpha, softplus)
        with torch.cuda.device(dev):
            st = lib.mmb_mmscan_bwd(desc, _lib.ptr(x), _lib.ptr(delta), _lib.ptr(A), _lib.ptr(B),
                                    _lib.ptr(C), _lib.ptr(D), _lib.ptr(z), _lib.ptr(delta_bias),
                                    _lib.ptr(ckpt), _lib.ptr(dout), _lib.ptr(dx), _lib.ptr(ddelta),
                                    _lib.ptr(dA), _lib.ptr(dB), _lib.ptr(dC), _lib.ptr(dD),
                                    _lib.ptr(dz), _lib.ptr(ddb), _lib.stream_of(x))
        _lib.check(st, "mmb_mmscan_bwd")
        if N != N0:
            dA, dB, dC = dA[:, :N0], dB[..., :N0], dC[..., :N0]
        need = ctx.needs_input_grad
        return (dx if need[0] else None, ddelta if need[1] else None, dA if need[2] else None,
                dB if need[3] else None, dC if need[4] else None,
                dD if need[5] else None, dz if need[6] else None, ddb if need[7] else None,
                None, None, None)


def selective_scan_momentum_fn(x, delta, A, B, C, D=None, z=None, delta_bias=None,
                               delta_softplus=False, beta=0.6, alpha=1.0):
    """Fused momentum selective scan; see the module docstring.  All tensors on one
    CUDA device; x, delta, z (batch, seqlen, dim); A (dim, d_state); B, C
    (batch, seqlen, d_state); D, delta_bias (dim).  Returns fp32 (batch, seqlen, dim)."""
    return SelectiveScanMomentumFn.apply(x, delta, A, B, C, D, z, delta_bias,
                                         bool(delta_softplus), float(beta), float(alpha))
