"""Drop-in for the reference's warp_momentum_scan_cuda module.

The reference's warp kernel evaluates the same recurrence as momentum_scan_cuda
in its 2x2 form  u_t = M_t u_{t-1} + F_t,  M_t = [[deltaA_t, beta], [0, beta]],
F_t = [u_t, u_t]  (warp_momentum_scan_cuda.py:34-126), so the forward here is
the same sm_100a row scan.  The reference's backward kernel
(warp_momentum_scan_cuda.py:130-230) is documented there as having correctness
issues; this module returns the exact adjoint instead, identical to
momentum_scan_cuda's:
    gh_t = g_t + deltaA_{t+1} gh_{t+1};  gv_t = gh_t + beta gv_{t+1};
    d momentum_input_t = gv_t;  d deltaA_t = gh_t h_{t-1}  (0 at t = 0).
"""
from __future__ import annotations

import torch

from . import _lib
from .momentum_scan_cuda import _as_rows, _rows_bwd, _rows_fwd


class WarpMomentumScanCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, deltaA, beta, momentum_input):
        a = _as_rows(deltaA)
        u = _as_rows(momentum_input)
        if a.shape != u.shape:
            raise ValueError("deltaA and momentum_input must have the same (rows, L) shape")
        h = torch.empty_like(u)
        _rows_fwd(a, beta, u, h)
        ctx.save_for_backward(a, h)
        ctx.beta = float(beta)
        return h

    @staticmethod
    def backward(ctx, grad_output):
        a, h = ctx.saved_tensors
        need_a, _, need_u = ctx.needs_input_grad
        da = torch.empty_like(a) if need_a else None
        du = torch.empty_like(a) if need_u else None
        if da is not None or du is not None:
            _rows_bwd(grad_output.float().contiguous(), a, ctx.beta, h, da, du)
        return da, None, du


warp_momentum_scan_cuda = WarpMomentumScanCUDA.apply


class _WarpKernel:
    """launch_warp_forward / launch_warp_backward of the reference extension
    (warp_momentum_scan_cuda.py:336-339).  The backward takes the gradient of the
    v states as absent (the reference's autograd always passes zeros there)."""

    @staticmethod
    def launch_warp_forward(A, F, beta, H_out, V_out):
        _rows_fwd(A, beta, F, H_out, V_out)

    @staticmethod
    def launch_warp_backward(grad_h_out, grad_v_out, A, F, beta, h_states, v_states, grad_A,
                             grad_F):
        _rows_bwd(grad_h_out, A, beta, h_states, grad_A, grad_F)


_kernel = _WarpKernel()


def load_warp_momentum_cuda():
    _lib.load()
    return _kernel


def get_warp_momentum_kernel():
    return load_warp_momentum_cuda()
