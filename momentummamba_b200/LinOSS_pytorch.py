"""LinOSS on the sm_100a kernels -- drop-in for the reference's LinOSS_pytorch.py.

Same names, module tree and parameter names.  The scan inside
apply_linoss_im_complex / apply_linoss_imex_complex runs on the fused LinOSS
kernel (transition and input scale built in registers per oscillator, chunked
over time, batched over sequences), so LinOSSLayer needs no vmap.  The complex
GEMMs around it (Bu = B u, y = Re(C x2) + D u, and their gradients) run on the
tensor cores (tc_gemm: tcgen05 with a 3 x tf32 split, fp32-grade accuracy) as
real GEMMs on interleaved complex data, so Bu comes out in the scan's layout
and x2 goes in as it is: no re/im copies, the feedthrough D u is the y GEMM's
epilogue.  ``parallel_scan_batched`` is the generic 2x2 scan kernel on one
sequence.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .scan2 import _DISC, _real_view, linoss_scan, scan2
from .tc_gemm import col_dot, gemm_nt, gemm_tn, split_tf32

VMAP_AVAILABLE = True


def simple_uniform_init(shape: Tuple[int, ...], std: float = 1.0) -> torch.Tensor:
    """U(-std, std) (LinOSS_pytorch.py:19-22)."""
    return torch.rand(shape) * 2.0 * std - std


class GLU(nn.Module):
    def __init__(self, input_dim: int, output_dim: int):
        super().__init__()
        self.w1 = nn.Linear(input_dim, output_dim, bias=True)
        self.w2 = nn.Linear(input_dim, output_dim, bias=True)

    def forward(self, x):
        return self.w1(x) * torch.sigmoid(self.w2(x))


def create_identity_padding(A_elements, b_elements, pad_length):
    """Identity transitions and zero inputs (LinOSS_pytorch.py:37-50)."""
    P = A_elements.shape[-1] // 4
    ident = torch.zeros(pad_length, 4 * P, device=A_elements.device)
    ident[..., :P] = 1.0
    ident[..., 3 * P:] = 1.0
    return ident, torch.zeros(pad_length, 2 * P, device=A_elements.device, dtype=b_elements.dtype)


def parallel_scan_batched(A_elements: torch.Tensor, b_elements: torch.Tensor):
    """Inclusive 2x2 scan of one sequence: A (L, 4P), b (L, 2P) real or complex ->
    (A_scan, b_scan) (LinOSS_pytorch.py:53-96)."""
    Ms, X = scan2(A_elements.unsqueeze(0), b_elements.unsqueeze(0))
    return Ms[0], X[0]


def binary_operator_batched(A_prev, b_prev, A_curr, b_curr):
    """(A_curr A_prev, A_curr b_prev + b_curr) on [A | B | C | D] blocks
    (LinOSS_pytorch.py:99-132)."""
    P = A_prev.shape[-1] // 4
    iA, iB, iC, iD = (A_prev[..., k * P:(k + 1) * P] for k in range(4))
    jA, jB, jC, jD = (A_curr[..., k * P:(k + 1) * P] for k in range(4))
    A_res = torch.cat([jA * iA + jB * iC, jA * iB + jB * iD, jC * iA + jD * iC, jC * iB + jD * iD],
                      dim=-1)
    b1, b2 = b_prev[..., :P], b_prev[..., P:]
    return A_res, torch.cat([jA * b1 + jB * b2, jC * b1 + jD * b2], dim=-1) + b_curr


def complex_matmul_real_input(B_real, B_imag, input_real):
    """(B_real + i B_imag) u for u (..., L, H) -> (re, im) each (..., L, P)."""
    return input_real @ B_real.t(), input_real @ B_imag.t()


def complex_matmul_complex_state(C_real, C_imag, state_real, state_imag):
    """Re(C x) for C (H, P), x (..., L, P) -> (..., L, H)."""
    return state_real @ C_real.t() - state_imag @ C_imag.t()


class LinOSSLayerFn(torch.autograd.Function):
    """y = Re(C x2) + D u with x2 the LinOSS scan of F(B u) (LinOSS_pytorch.py:153-239,
    :306-312), on interleaved complex data: Bm = [B_re; B_im] rows interleaved
    (2P, H), Cc[h, (p, re | im)] = (C_re, -C_im)[h, p] (H, 2P), so that
    Bu = u Bm^T comes out as complex (B, L, P) and y = x2 Cc^T + D u reads x2 as
    it is.  Gradients: dx2 = dy Cc, dBu from the scan's adjoint, du = dBu Bm +
    D dy, dBm = dBu^T u, dCc = dy^T x2, dD = sum dy u."""

    @staticmethod
    def forward(ctx, disc, A_diag, step, B_real, B_imag, C_real, C_imag, D, u):
        _lib.require_cuda(A_diag, step, B_real, B_imag, C_real, C_imag, D, u)
        if disc not in _DISC:
            raise ValueError(f"Discretization type {disc} not implemented")
        Bsz, L, H = u.shape
        P = A_diag.shape[0]
        u2 = u.reshape(Bsz * L, H).float().contiguous()
        Bm = torch.stack([B_real.float(), B_imag.float()], dim=1).reshape(2 * P, H)
        Cc = torch.stack([C_real.float(), -C_imag.float()], dim=2).reshape(H, 2 * P)
        Bu = gemm_nt(u2, split_tf32(Bm)).view(Bsz, L, P, 2)
        A, s = A_diag.float().contiguous(), step.float().contiguous()
        lib = _lib.load()
        x2 = torch.empty_like(Bu)
        work = torch.empty(lib.mmb_linoss_work_floats(Bsz, L, P), device=u.device)
        with torch.cuda.device(u.device):
            st = lib.mmb_linoss_fwd(_DISC[disc], Bsz, L, P, _lib.ptr(A), _lib.ptr(s),
                                    _lib.ptr(Bu), _lib.ptr(x2), _lib.ptr(work),
                                    _lib.stream_of(u))
        _lib.check(st, "mmb_linoss_fwd")
        Dv = D.float().contiguous() if D is not None else None
        y = gemm_nt(x2.view(Bsz * L, 2 * P), split_tf32(Cc), E=u2 if Dv is not None else None,
                    evec=Dv)
        ctx.save_for_backward(A, s, Bm, Cc, u2, Bu, x2, work, Dv)
        ctx.disc, ctx.has_d, ctx.shape = disc, Dv is not None, (Bsz, L, H, P)
        return y.view(Bsz, L, H)

    @staticmethod
    def backward(ctx, dy):
        A, s, Bm, Cc, u2, Bu, x2, work, Dv = ctx.saved_tensors
        Bsz, L, H, P = ctx.shape
        dy2 = dy.reshape(Bsz * L, H).float().contiguous()
        dx2 = gemm_nt(dy2, split_tf32(Cc.t()))                     # (B L, 2P)
        lib = _lib.load()
        dBu = torch.empty_like(Bu)
        dA = torch.empty_like(A)
        ds = torch.empty_like(s)
        with torch.cuda.device(A.device):
            st = lib.mmb_linoss_bwd(_DISC[ctx.disc], Bsz, L, P, _lib.ptr(A), _lib.ptr(s),
                                    _lib.ptr(Bu), _lib.ptr(dx2), _lib.ptr(dBu), _lib.ptr(dA),
                                    _lib.ptr(ds), _lib.ptr(work), _lib.stream_of(A))
        _lib.check(st, "mmb_linoss_bwd")
        dBu2 = dBu.view(Bsz * L, 2 * P)
        du = gemm_nt(dBu2, split_tf32(Bm.t()), E=dy2 if ctx.has_d else None,
                     evec=Dv if ctx.has_d else None)
        dBm = gemm_tn(dBu2, u2)                                     # (2P, H)
        dCc = gemm_tn(dy2, x2.view(Bsz * L, 2 * P))                 # (H, 2P)
        dD = (col_dot(dy2, u2) if H % 4 == 0 else (dy2 * u2).sum(0)) if ctx.has_d else None
        dBm = dBm.view(P, 2, H)
        dCc = dCc.view(H, P, 2)
        return (None, dA, ds, dBm[:, 0], dBm[:, 1], dCc[..., 0], -dCc[..., 1], dD,
                du.view(Bsz, L, H))


def _apply(disc, A_diag, B_real, B_imag, C_real, C_imag, input_sequence, step, D=None):
    squeeze = input_sequence.dim() == 2
    u = input_sequence.unsqueeze(0) if squeeze else input_sequence
    y = LinOSSLayerFn.apply(disc, A_diag, step, B_real, B_imag, C_real, C_imag, D, u)
    return y[0] if squeeze else y


def apply_linoss_im_complex(A_diag, B_real, B_imag, C_real, C_imag, input_sequence, step):
    """LinOSS-IM (LinOSS_pytorch.py:153-195); input (L, H) or batched (B, L, H)."""
    return _apply("IM", A_diag, B_real, B_imag, C_real, C_imag, input_sequence, step)


def apply_linoss_imex_complex(A_diag, B_real, B_imag, C_real, C_imag, input_sequence, step):
    """LinOSS-IMEX (LinOSS_pytorch.py:198-239); input (L, H) or batched (B, L, H)."""
    return _apply("IMEX", A_diag, B_real, B_imag, C_real, C_imag, input_sequence, step)


class LinOSSLayer(nn.Module):
    def __init__(self, ssm_size: int, H: int, discretization: str):
        super().__init__()
        self.discretization = discretization
        self.A_diag = nn.Parameter(torch.rand(ssm_size))
        self.B_real = nn.Parameter(simple_uniform_init((ssm_size, H), std=1.0 / math.sqrt(H)))
        self.B_imag = nn.Parameter(simple_uniform_init((ssm_size, H), std=1.0 / math.sqrt(H)))
        self.C_real = nn.Parameter(simple_uniform_init((H, ssm_size), std=1.0 / math.sqrt(ssm_size)))
        self.C_imag = nn.Parameter(simple_uniform_init((H, ssm_size), std=1.0 / math.sqrt(ssm_size)))
        self.D = nn.Parameter(torch.randn(H))
        self.steps = nn.Parameter(torch.rand(ssm_size))

    def forward(self, input_sequence):
        if input_sequence.dim() not in (2, 3):
            raise ValueError(f"Input must be 2D (L, H) or 3D (B, L, H), got {input_sequence.dim()}D")
        if self.discretization not in ("IM", "IMEX"):
            raise ValueError(f"Discretization type {self.discretization} not implemented")
        A = F.relu(self.A_diag)
        steps = torch.sigmoid(self.steps)
        # the feedthrough D u is the output GEMM's epilogue
        return _apply(self.discretization, A, self.B_real, self.B_imag, self.C_real, self.C_imag,
                      input_sequence, steps, D=self.D)


class LinOSSBlock(nn.Module):
    def __init__(self, ssm_size: int, H: int, discretization: str, drop_rate: float = 0.05,
                 norm_type: str = "batch"):
        super().__init__()
        self.norm_type = norm_type
        self.H = H
        if norm_type == "batch":
            self.norm = nn.GroupNorm(num_groups=H, num_channels=H, affine=False)
        elif norm_type == "layer":
            self.norm = nn.LayerNorm(H, elementwise_affine=False)
        else:
            raise ValueError(f"norm_type must be 'batch' or 'layer', got {norm_type}")
        self.ssm = LinOSSLayer(ssm_size, H, discretization)
        self.glu = GLU(H, H)
        self.dropout = nn.Dropout(p=drop_rate)

    def forward(self, x):
        skip = x
        if self.norm_type == "batch":
            if x.dim() == 2:
                x = self.norm(x.t().unsqueeze(0)).squeeze(0).t()
            else:
                x = self.norm(x.transpose(1, 2)).transpose(1, 2)
        else:
            x = self.norm(x)
        x = self.ssm(x)
        x = self.dropout(F.gelu(x))
        x = self.glu(x)
        x = self.dropout(x)
        return skip + x


class LinOSS(nn.Module):
    def __init__(self, num_blocks: int, N: int, ssm_size: int, H: int, output_dim: int,
                 classification: bool, output_step: int, discretization: str,
                 norm_type: str = "batch"):
        super().__init__()
        self.classification = classification
        self.output_step = output_step
        self.linear_encoder = nn.Linear(N, H)
        self.blocks = nn.ModuleList([LinOSSBlock(ssm_size, H, discretization, norm_type=norm_type)
                                     for _ in range(num_blocks)])
        self.linear_layer = nn.Linear(H, output_dim)

    def forward(self, x):
        x = self.linear_encoder(x)
        for block in self.blocks:
            x = block(x)
        if self.classification:
            x = x.mean(dim=0) if x.dim() == 2 else x.mean(dim=1)
            return self.linear_layer(x)
        x = x[..., self.output_step - 1::self.output_step, :]
        return torch.tanh(self.linear_layer(x))
