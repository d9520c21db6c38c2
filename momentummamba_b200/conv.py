"""The momentum block's producer and decode step on the sm_100a kernels.

* ``conv1d_silu(x, weight, bias)``: causal depthwise conv1d + SiLU over time on
  (B, L, D) activations -- the block's x branch,
  ``silu(conv1d(x.transpose(1, 2))[:, :, :L].transpose(1, 2))``
  (mamba_momentum.py:217-223) -- in one pass without the transposes, with its
  backward (dx, dweight, dbias).
* ``conv1d_step`` / ``mmscan_step``: the decode-time conv-cache update
  (mamba_momentum.py:455-459, :466) and the single-token momentum state update
  with the dt softplus and the SiLU(z) gate fused (:473-515, :461-464).

fp32 arithmetic; other dtypes are computed in fp32 and cast back.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


def _f32(t):
    return None if t is None else t.float()


class Conv1dSiluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, state_in):
        _lib.require_cuda(x, weight, bias, state_in)
        lib = _lib.load()
        in_dtype = x.dtype
        x = _f32(x)
        if x.stride(-1) != 1:
            x = x.contiguous()
        Bsz, L, D = x.shape
        W = weight.shape[-1]
        w = _f32(weight).reshape(D, W).contiguous()
        b = None if bias is None else _f32(bias).contiguous()
        s_in = None if state_in is None else _f32(state_in).contiguous()
        out = torch.empty((Bsz, L, D), device=x.device, dtype=torch.float32)
        xs = (ctypes.c_int64 * 2)(x.stride(0), x.stride(1))
        with torch.cuda.device(x.device):
            st = lib.mmb_conv1d_silu_fwd(Bsz, L, D, W, _lib.ptr(x), xs, _lib.ptr(w), _lib.ptr(b),
                                         _lib.ptr(s_in), None, _lib.ptr(out), _lib.stream_of(x))
        _lib.check(st, "mmb_conv1d_silu_fwd")
        ctx.save_for_backward(x, w, b, s_in)
        ctx.meta = (in_dtype, weight.shape, weight.dtype, None if bias is None else bias.dtype)
        return out if in_dtype == torch.float32 else out.to(in_dtype)

    @staticmethod
    def backward(ctx, dout):
        lib = _lib.load()
        x, w, b, s_in = ctx.saved_tensors
        in_dtype, wshape, wdtype, bdtype = ctx.meta
        Bsz, L, D = x.shape
        W = w.shape[1]
        dout = dout.float().contiguous()
        dx = torch.empty((Bsz, L, D), device=x.device, dtype=torch.float32)
        dw = torch.empty((D, W), device=x.device, dtype=torch.float32)
        db = torch.empty((D,), device=x.device, dtype=torch.float32) if b is not None else None
        xs = (ctypes.c_int64 * 2)(x.stride(0), x.stride(1))
        with torch.cuda.device(x.device):
            st = lib.mmb_conv1d_silu_bwd(Bsz, L, D, W, _lib.ptr(x), xs, _lib.ptr(w), _lib.ptr(b),
                                         _lib.ptr(s_in), _lib.ptr(dout), _lib.ptr(dx), _lib.ptr(dw),
                                         _lib.ptr(db), _lib.stream_of(x))
        _lib.check(st, "mmb_conv1d_silu_bwd")
        need = ctx.needs_input_grad
        return (dx.to(in_dtype) if need[0] else None,
                dw.reshape(wshape).to(wdtype) if need[1] else None,
                db.to(bdtype) if (need[2] and db is not None) else None, None)


def conv1d_silu(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                state_in: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(causal depthwise conv1d(x)) for x (B, L, D), weight (D, 1, W) or (D, W),
    bias (D); state_in (B, D, W-1) holds the inputs before t = 0 (zeros if None)."""
    return Conv1dSiluFn.apply(x, weight, bias, state_in)


def conv1d_silu_state(x: torch.Tensor, weight: torch.Tensor, bias=None, state_in=None):
    """Inference prefill: (out, state_out) with state_out (B, D, W-1) the last
    W-1 inputs, the decode cache for conv1d_step."""
    _lib.require_cuda(x, weight, bias, state_in)
    lib = _lib.load()
    x = _f32(x)
    if x.stride(-1) != 1:
        x = x.contiguous()
    Bsz, L, D = x.shape
    W = weight.shape[-1]
    w = _f32(weight).reshape(D, W).contiguous()
    b = None if bias is None else _f32(bias).contiguous()
    s_in = None if state_in is None else _f32(state_in).contiguous()
    out = torch.empty((Bsz, L, D), device=x.device)
    s_out = torch.empty((Bsz, D, W - 1), device=x.device)
    xs = (ctypes.c_int64 * 2)(x.stride(0), x.stride(1))
    with torch.cuda.device(x.device):
        st = lib.mmb_conv1d_silu_fwd(Bsz, L, D, W, _lib.ptr(x), xs, _lib.ptr(w), _lib.ptr(b),
                                     _lib.ptr(s_in), _lib.ptr(s_out), _lib.ptr(out),
                                     _lib.stream_of(x))
    _lib.check(st, "mmb_conv1d_silu_fwd")
    return out, s_out


def conv1d_step(x: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor,
                bias: Optional[torch.Tensor] = None, out_state: Optional[torch.Tensor] = None):
    """One token: (silu(conv over [conv_state | x]), new conv state).  conv_state
    (B, D, W-1); the new state is written to out_state (may be conv_state itself;
    a new tensor when None).  x (B, D) rows with unit column stride."""
    _lib.require_cuda(x, conv_state, weight, bias, out_state)
    x = _f32(x)
    if x.stride(-1) != 1:
        x = x.contiguous()
    Bsz, D = x.shape
    W = weight.shape[-1]
    s_in = _f32(conv_state).contiguous()
    if out_state is None:
        out_state = torch.empty_like(s_in)
    elif out_state.dtype != torch.float32 or not out_state.is_contiguous():
        raise ValueError("out_state must be a contiguous fp32 tensor")
    w = _f32(weight).reshape(D, W).contiguous()
    b = None if bias is None else _f32(bias).contiguous()
    out = torch.empty((Bsz, D), device=x.device)
    with torch.cuda.device(x.device):
        st = _lib.load().mmb_conv1d_step(Bsz, D, W, _lib.ptr(x), x.stride(0), _lib.ptr(s_in),
                                         _lib.ptr(out_state), _lib.ptr(w), _lib.ptr(b),
                                         _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "mmb_conv1d_step")
    return out, out_state


def mmscan_step(x, delta, A, B, C, h=None, v=None, D=None, z=None, delta_bias=None,
                delta_softplus=False, beta=0.6, alpha=1.0, h_out=None, v_out=None):
    """One token of the momentum scan.  h, v (B, D, N) the state before it (None =
    zeros); the state after goes to h_out, v_out (may be h, v themselves; new
    tensors when None).  x, delta, z (B, D); B, C (B, N) (row strides allowed);
    A (D, N); D, delta_bias (D).  Returns ((C.h + D x) * silu(z), h_out, v_out)
    (no gate when z is None)."""
    _lib.require_cuda(x, delta, A, B, C, h, v, D, z, delta_bias, h_out, v_out)

    def row(t):
        t = _f32(t)
        return t if t.stride(-1) == 1 else t.contiguous()

    x, delta, B, C, z = (None if t is None else row(t) for t in (x, delta, B, C, z))
    A = _f32(A).contiguous()
    D = None if D is None else _f32(D).contiguous()
    delta_bias = None if delta_bias is None else _f32(delta_bias).contiguous()
    Bsz, Dm = x.shape
    N = A.shape[1]
    h = None if h is None else _f32(h).contiguous()
    v = None if v is None else _f32(v).contiguous()
    if h_out is None:
        h_out = torch.empty((Bsz, Dm, N), device=x.device)
    if v_out is None:
        v_out = torch.empty((Bsz, Dm, N), device=x.device)
    for t in (h, v, h_out, v_out):
        if t is not None and (t.dtype != torch.float32 or t.shape != (Bsz, Dm, N)
                              or not t.is_contiguous()):
            raise ValueError("states must be contiguous fp32 (batch, dim, d_state) tensors")
    d = _lib.StepDesc()
    d.batch, d.dim, d.dstate = Bsz, Dm, N
    d.x_row_stride, d.delta_row_stride = x.stride(0), delta.stride(0)
    d.z_row_stride = z.stride(0) if z is not None else 0
    d.B_row_stride, d.C_row_stride = B.stride(0), C.stride(0)
    d.state_stride[:] = (Dm * N, N)
    d.beta, d.alpha = float(beta), float(alpha)
    d.delta_softplus = 1 if delta_softplus else 0
    out = torch.empty((Bsz, Dm), device=x.device)
    with torch.cuda.device(x.device):
        st = _lib.load().mmb_mmscan_step(ctypes.byref(d), _lib.ptr(x), _lib.ptr(delta), _lib.ptr(A),
                                         _lib.ptr(B), _lib.ptr(C), _lib.ptr(D), _lib.ptr(z),
                                         _lib.ptr(delta_bias), _lib.ptr(h), _lib.ptr(v),
                                         _lib.ptr(h_out), _lib.ptr(v_out), _lib.ptr(out),
                                         _lib.stream_of(x))
    _lib.check(st, "mmb_mmscan_step")
    return out, h_out, v_out
