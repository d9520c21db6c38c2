"""LinOSS on the sm_100a scan kernels -- drop-in for the reference's LinOSS_pytorch.py.

Same names, module tree and parameter names.  The scan inside
apply_linoss_im_complex / apply_linoss_imex_complex runs on the fused LinOSS
kernel (transition and input scale built in registers per oscillator, chunked
over time, batched over sequences), so LinOSSLayer needs no vmap; the complex
GEMMs around it (Bu = B u, y = Re(C x2)) stay with cuBLAS.
``parallel_scan_batched`` is the generic 2x2 scan kernel on one sequence.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .scan2 import linoss_scan, scan2

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


def _apply(disc, A_diag, B_real, B_imag, C_real, C_imag, input_sequence, step):
    squeeze = input_sequence.dim() == 2
    u = input_sequence.unsqueeze(0) if squeeze else input_sequence
    bu_r, bu_i = complex_matmul_real_input(B_real, B_imag, u.float())
    x2 = linoss_scan(disc, A_diag, step, torch.complex(bu_r, bu_i))
    y = complex_matmul_complex_state(C_real, C_imag, x2.real, x2.imag)
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
        ys = _apply(self.discretization, A, self.B_real, self.B_imag, self.C_real, self.C_imag,
                    input_sequence, steps)
        return ys + input_sequence * self.D


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
