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

Activations (x, delta, z, B, C) are fp32 or, when all of them are bf16, bf16:
then out and the activation gradients are bf16 too, while the state, the
arithmetic and every sum stay fp32 (the reference up-casts everything to fp32,
momentum_scan_cuda.py:215-216; bf16 halves the activation traffic).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_SUPPORTED_N = (8, 16, 32, 64)


def _padded_state(N: int) -> int:
    for n in _SUPPORTED_N:
        if N <= n:
            return n
    raise RuntimeError(f"momentummamba_b200: d_state={N} > 64 is not supported")


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


def _bf16_ok(ts) -> bool:
    """bf16 kernels need 16-byte aligned rows: pointers, dim and strides in units of 8."""
    for t in ts:
        if t is None:
            continue
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.data_ptr() % 16:
            return False
        if t.shape[-1] % 8 or t.stride(0) % 8 or t.stride(1) % 8:
            return False
    return True


class ScanCall:
    """One momentum-scan problem packed for the C ABI: activation dtype chosen,
    fp32 parameters, d_state padded to a compiled size, descriptor built."""

    def __init__(self, x, delta, A, B, C, D=None, z=None, delta_bias=None,
                 delta_softplus=False, beta=0.6, alpha=1.0, time_chunk=0):
        _lib.require_cuda(x, delta, A, B, C, D, z, delta_bias)
        self.N0 = A.shape[1]
        N = _padded_state(self.N0)
        acts = [x, delta, z, B, C]
        bf16 = all(t is None or t.dtype == torch.bfloat16 for t in acts) and _bf16_ok(
            [x, delta, z] + ([B, C] if N == self.N0 else []))
        adt = torch.bfloat16 if bf16 else torch.float32

        def act(t):
            if t is None:
                return None
            if t.dtype != adt:
                t = t.to(adt)
            return t if t.stride(-1) == 1 else t.contiguous()

        x, delta, z, B, C = (act(t) for t in acts)
        f32 = lambda t: None if t is None else t.float().contiguous()
        A, D, delta_bias = f32(A), f32(D), f32(delta_bias)
        if N != self.N0:
            A, B, C = _pad_last(A, N), _pad_last(B, N), _pad_last(C, N)
        Bsz, L, Dm = x.shape
        if delta.shape != x.shape or (z is not None and z.shape != x.shape):
            raise ValueError("x, delta and z must share the shape (batch, seqlen, dim)")
        if A.shape[0] != Dm or B.shape != (Bsz, L, N) or C.shape != (Bsz, L, N):
            raise ValueError("A must be (dim, d_state); B and C (batch, seqlen, d_state)")
        self.x, self.delta, self.z, self.B, self.C = x, delta, z, B, C
        self.A, self.D, self.delta_bias = A, D, delta_bias
        self.N, self.shape, self.adtype = N, (Bsz, L, Dm), adt
        self.softplus, self.beta, self.alpha = bool(delta_softplus), float(beta), float(alpha)
        d = _lib.MMScanDesc()
        d.batch, d.seqlen, d.dim = Bsz, L, Dm
        d.dstate = N
        d.x_stride[:] = _strides(x)
        d.delta_stride[:] = _strides(delta)
        d.z_stride[:] = _strides(z)
        d.B_stride[:] = _strides(B)
        d.C_stride[:] = _strides(C)
        d.beta, d.alpha = self.beta, self.alpha
        d.delta_softplus = 1 if delta_softplus else 0
        d.dtype = _lib.MMB_BF16 if bf16 else _lib.MMB_F32
        d.time_chunk = int(time_chunk)
        self.desc = d

    @property
    def device(self):
        return self.x.device

    def state_shape(self, k: int = 2):
        Bsz, _, Dm = self.shape
        return (Bsz, Dm, k, self.N)

    def tensors(self, **extra) -> _lib.MMScanTensors:
        t = _lib.MMScanTensors()
        for name, v in (("x", self.x), ("delta", self.delta), ("z", self.z), ("B", self.B),
                        ("C", self.C), ("A", self.A), ("D", self.D),
                        ("delta_bias", self.delta_bias), *extra.items()):
            setattr(t, name, None if v is None else v.data_ptr())
        return t

    def _run(self, fn, what, *args):
        lib = _lib.load()
        with torch.cuda.device(self.device):
            st = getattr(lib, fn)(ctypes.byref(self.desc), *args, _lib.stream_of(self.x))
        _lib.check(st, what)

    # -- the four per-call operations --------------------------------------
    def forward(self, need_ckpt: bool, state_in=None, want_state=False):
        lib = _lib.load()
        Bsz, L, Dm = self.shape
        out = torch.empty(self.shape, device=self.device, dtype=self.adtype)
        ckpt = None
        if need_ckpt:
            ckpt = torch.empty(lib.mmb_mmscan_workspace_floats(ctypes.byref(self.desc)),
                               device=self.device, dtype=torch.float32)
        state_out = torch.empty(self.state_shape(), device=self.device) if want_state else None
        t = self.tensors(out=out, ckpt=ckpt, state_in=state_in, state_out=state_out)
        self._run("mmb_mmscan_forward", "mmb_mmscan_forward", ctypes.byref(t))
        return out, ckpt, state_out

    def backward(self, ckpt, dout, gstate_in=None, want_gstate=False):
        Bsz, L, Dm = self.shape
        dev, f32 = self.device, torch.float32
        dout = dout.to(self.adtype).contiguous()
        dx = torch.empty(self.shape, device=dev, dtype=self.adtype)
        ddelta = torch.empty(self.shape, device=dev, dtype=self.adtype)
        dz = torch.empty(self.shape, device=dev, dtype=self.adtype) if self.z is not None else None
        dA = torch.empty((Dm, self.N), device=dev, dtype=f32)
        dB = torch.empty((Bsz, L, self.N), device=dev, dtype=f32)
        dC = torch.empty((Bsz, L, self.N), device=dev, dtype=f32)
        dD = torch.empty((Dm,), device=dev, dtype=f32) if self.D is not None else None
        ddb = torch.empty((Dm,), device=dev, dtype=f32) if self.delta_bias is not None else None
        gout = torch.empty(self.state_shape(), device=dev) if want_gstate else None
        t = self.tensors(ckpt=ckpt, dout=dout, gstate_in=gstate_in, dx=dx, ddelta=ddelta, dz=dz,
                         dA=dA, dB=dB, dC=dC, dD=dD, ddelta_bias=ddb, gstate_out=gout)
        self._run("mmb_mmscan_backward", "mmb_mmscan_backward", ctypes.byref(t))
        if self.N != self.N0:
            dA, dB, dC = dA[:, : self.N0], dB[..., : self.N0], dC[..., : self.N0]
        return dx, ddelta, dA, dB, dC, dD, dz, ddb, gout

    def fwd_summary(self):
        summ = torch.empty(self.state_shape(4), device=self.device)
        t = self.tensors()
        self._run("mmb_mmscan_fwd_summary", "mmb_mmscan_fwd_summary", ctypes.byref(t),
                  _lib.ptr(summ))
        return summ

    def bwd_summary(self, dout):
        gsumm = torch.empty(self.state_shape(2), device=self.device)
        dout = dout.to(self.adtype).contiguous()  # kept alive until the launch
        t = self.tensors(dout=dout)
        self._run("mmb_mmscan_bwd_summary", "mmb_mmscan_bwd_summary", ctypes.byref(t),
                  _lib.ptr(gsumm))
        return gsumm


def _cast_like(g, ref):
    if g is None or ref is None:
        return g
    return g if g.dtype == ref.dtype else g.to(ref.dtype)


class SelectiveScanMomentumFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, delta, A, B, C, D, z, delta_bias, delta_softplus, beta, alpha,
                time_chunk=0):
        call = ScanCall(x, delta, A, B, C, D, z, delta_bias, delta_softplus, beta, alpha,
                        time_chunk)
        need_grad = any(ctx.needs_input_grad[:8])
        out, ckpt, _ = call.forward(need_grad)
        ctx.call, ctx.ckpt = call, ckpt
        ctx.in_dtypes = [None if t is None else t.dtype
                         for t in (x, delta, A, B, C, D, z, delta_bias)]
        return out

    @staticmethod
    def backward(ctx, dout):
        call = ctx.call
        grads = call.backward(ctx.ckpt, dout)[:8]
        dx, ddelta, dA, dB, dC, dD, dz, ddb = grads
        order = (dx, ddelta, dA, dB, dC, dD, dz, ddb)
        res = []
        for need, g, dt in zip(ctx.needs_input_grad[:8], order, ctx.in_dtypes):
            res.append((g if dt is None or g.dtype == dt else g.to(dt)) if need and g is not None
                       else None)
        ctx.call = ctx.ckpt = None
        return (*res, None, None, None, None)


def selective_scan_momentum_fn(x, delta, A, B, C, D=None, z=None, delta_bias=None,
                               delta_softplus=False, beta=0.6, alpha=1.0, time_chunk=0):
    """Fused momentum selective scan; see the module docstring.  All tensors on one
    CUDA device; x, delta, z (batch, seqlen, dim); A (dim, d_state); B, C
    (batch, seqlen, d_state); D, delta_bias (dim).  Returns (batch, seqlen, dim)
    in the activation dtype (bf16 when x, delta, z, B, C are all bf16, else fp32).
    time_chunk: steps per time chunk scanned by separate CTAs (0: the library
    splits short batches of long sequences on its own; < 0: never split)."""
    return SelectiveScanMomentumFn.apply(x, delta, A, B, C, D, z, delta_bias,
                                         bool(delta_softplus), float(beta), float(alpha),
                                         int(time_chunk))
