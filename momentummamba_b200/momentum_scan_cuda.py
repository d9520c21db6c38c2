"""Drop-in for the reference's momentum_scan_cuda module (momentum_scan_cuda.py).

``momentum_scan_cuda(deltaA, beta, momentum_input)`` scans rows of (R, L)
tensors:  v_t = beta*v_{t-1} + u_t ;  h_t = deltaA_t*h_{t-1} + v_t, returning h.
Backward (momentum_scan_cuda.py:231-251): (grad_deltaA, None, grad_input), with
grad_deltaA zero at t = 0 and None for inputs that do not require grad.

``get_momentum_kernel()`` returns an object with the reference extension's two
launchers, ``launch_forward(deltaA, beta, input, output_h)`` and
``launch_backward(grad_output, deltaA, beta, output_h, grad_deltaA, grad_input)``
(momentum_scan_cuda.py:175-178), writing into the given tensors in place and
skipping empty gradient tensors, but on the current stream without a device-wide
synchronisation.
"""
from __future__ import annotations

import torch

from . import _lib


def _rows_fwd(deltaA, beta, u, h, v=None):
    _lib.require_cuda(deltaA, u, h, v)
    lib = _lib.load()
    R, L = deltaA.shape
    with torch.cuda.device(deltaA.device):
        st = lib.mmb_rows_fwd(R, L, _lib.ptr(deltaA), float(beta), _lib.ptr(u), _lib.ptr(h),
                              _lib.ptr(v), _lib.stream_of(deltaA))
    _lib.check(st, "mmb_rows_fwd")


def _rows_bwd(g, deltaA, beta, h, da, du):
    _lib.require_cuda(g, deltaA, h, da, du)
    lib = _lib.load()
    R, L = deltaA.shape
    with torch.cuda.device(deltaA.device):
        st = lib.mmb_rows_bwd(R, L, _lib.ptr(g), _lib.ptr(deltaA), float(beta), _lib.ptr(h),
                              _lib.ptr(da), _lib.ptr(du), _lib.stream_of(deltaA))
    _lib.check(st, "mmb_rows_bwd")


def _as_rows(t: torch.Tensor) -> torch.Tensor:
    if t.dim() != 2:
        raise ValueError(f"expected a (rows, L) tensor, got shape {tuple(t.shape)}")
    return t.float().contiguous()


class MomentumScanCUDA(torch.autograd.Function):
    """Row momentum scan with autograd (momentum_scan_cuda.py:204-251)."""

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


momentum_scan_cuda = MomentumScanCUDA.apply


class _RowKernel:
    """The two launchers of the reference extension, on the sm_100a kernels."""

    @staticmethod
    def launch_forward(deltaA, beta, input, output_h):
        _rows_fwd(deltaA, beta, input, output_h)

    @staticmethod
    def launch_backward(grad_output, deltaA, beta, output_h, grad_deltaA, grad_input):
        da = grad_deltaA if grad_deltaA.numel() > 0 else None
        du = grad_input if grad_input.numel() > 0 else None
        if da is not None or du is not None:
            _rows_bwd(grad_output, deltaA, beta, output_h, da, du)


_kernel = _RowKernel()


def load_momentum_cuda():
    """Load the extension (the in-tree C-ABI library); raises if it is missing."""
    _lib.load()
    return _kernel


def get_momentum_kernel():
    return load_momentum_cuda()
