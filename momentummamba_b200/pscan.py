"""Drop-in for the reference's pscan module (pscan.py:21-234).

``pscan(A_in, X_in)`` returns H with H_t = A_t * H_{t-1} + X_t along dim 1 of
(B, L, D, N) tensors (any trailing shape); backward returns (gradA, gradX) with
gradA_t = H_{t-1} * gradX_t, zero at t = 0 (pscan.py:197-232).  Any L works
directly -- nothing is padded to a power of two.  ``npo2`` and ``pad_npo2`` are
kept with the reference's meaning for code that imports them.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _lib


def npo2(len):
    """Next power of two >= len (pscan.py:21-26)."""
    return 2 ** math.ceil(math.log2(len))


def pad_npo2(X):
    """Zero-pad dim 1 of (B, L, D, N) up to npo2(L) (pscan.py:28-41)."""
    len_npo2 = npo2(X.size(1))
    pad_tuple = (0, 0, 0, 0, 0, len_npo2 - X.size(1))
    return F.pad(X, pad_tuple, "constant", 0)


def _flat(t: torch.Tensor) -> torch.Tensor:
    return t.float().contiguous().reshape(t.shape[0], t.shape[1], -1)


class PScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A_in, X_in):
        _lib.require_cuda(A_in, X_in)
        if A_in.shape != X_in.shape or A_in.dim() < 2:
            raise ValueError("A_in and X_in must share a (B, L, ...) shape")
        A = _flat(A_in)
        X = _flat(X_in)
        Bsz, L, M = A.shape
        H = torch.empty_like(A)
        lib = _lib.load()
        with torch.cuda.device(A.device):
            st = lib.mmb_pscan_fwd(Bsz, L, M, _lib.ptr(A), _lib.ptr(X), _lib.ptr(H),
                                   _lib.stream_of(A))
        _lib.check(st, "mmb_pscan_fwd")
        ctx.save_for_backward(A, H)
        ctx.shape = A_in.shape
        return H.reshape(A_in.shape)

    @staticmethod
    def backward(ctx, grad_output_in):
        A, H = ctx.saved_tensors
        G = _flat(grad_output_in)
        Bsz, L, M = A.shape
        need_a, need_x = ctx.needs_input_grad
        dA = torch.empty_like(A) if need_a else None
        dX = torch.empty_like(A) if need_x else None
        if dA is not None or dX is not None:
            lib = _lib.load()
            with torch.cuda.device(A.device):
                st = lib.mmb_pscan_bwd(Bsz, L, M, _lib.ptr(A), _lib.ptr(H), _lib.ptr(G),
                                       _lib.ptr(dA), _lib.ptr(dX), _lib.stream_of(A))
            _lib.check(st, "mmb_pscan_bwd")
        shp = ctx.shape
        return (None if dA is None else dA.reshape(shp), None if dX is None else dX.reshape(shp))


pscan = PScan.apply
