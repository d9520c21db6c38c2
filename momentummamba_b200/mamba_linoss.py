"""Mamba-LinOSS on the sm_100a scan kernels -- drop-in for the reference's mamba_linoss.py.

Same configuration dataclass, module tree, parameter names and function names.
Every scan entry point -- parallel_scan_batched_complex,
parallel_scan_batched_complex_optimized, apply_scan_vmap -- runs the chunked
sm_100a 2x2 scan and returns the exact inclusive scan (A_scan, b_scan) with
gradients.  In the reference only the first is a correct scan; the 'optimized'
Blelloch variant and the default 'vmap' variant (up-sweep only) return wrong
states for longer sequences (mamba_linoss.py:484-558, :702-763), so results
here match the reference's 'vectorized' scan whatever scan_algorithm says.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .LinOSS_pytorch import binary_operator_batched
from .scan2 import linoss_selective, scan2

VMAP_AVAILABLE = True
torch_vmap = torch.func.vmap


@dataclass
class MambaLinOSSConfig:
    d_model: int
    n_layer: int
    d_state: int = 64
    linoss_discretization: str = "IM"
    a_init_method: str = "uniform"
    dt_min: float = 0.001
    dt_max: float = 0.1
    dt_init_floor: float = 1e-4
    expand_factor: int = 2
    d_conv: int = 4
    rms_norm_eps: float = 1e-5
    bias: bool = False
    conv_bias: bool = True
    dropout_rate: float = 0
    scan_algorithm: str = "vmap"
    use_vmap: bool = True

    def __post_init__(self):
        self.d_inner = self.expand_factor * self.d_model
        if self.linoss_discretization not in ["IM", "IMEX"]:
            raise ValueError(f"linoss_discretization must be 'IM' or 'IMEX', got {self.linoss_discretization}")
        if self.a_init_method not in ["log_uniform", "uniform", "relu"]:
            raise ValueError(f"a_init_method must be 'log_uniform', 'uniform', or 'relu', got {self.a_init_method}")
        if self.dt_min >= self.dt_max:
            raise ValueError(f"dt_min ({self.dt_min}) must be less than dt_max ({self.dt_max})")
        if self.scan_algorithm not in ["auto", "vectorized", "optimized", "vmap"]:
            raise ValueError("scan_algorithm must be one of ['auto', 'vectorized', 'optimized', 'vmap'], "
                             f"got {self.scan_algorithm}")
        if self.scan_algorithm == "auto":
            self.scan_algorithm = "vmap" if (self.use_vmap and VMAP_AVAILABLE) else "optimized"


class RMSNorm(nn.Module):
    def __init__(self, d_model: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model))

    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


class MambaLinOSS(nn.Module):
    def __init__(self, config: MambaLinOSSConfig):
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([MambaLinOSSBlock(config) for _ in range(config.n_layer)])
        self.norm_f = RMSNorm(config.d_model)

    def forward(self, x):
        for layer in self.layers:
            x = x + layer(x)
        return self.norm_f(x)


class MambaLinOSSBlock(nn.Module):
    def __init__(self, config: MambaLinOSSConfig):
        super().__init__()
        self.config = config
        self.in_proj = nn.Linear(config.d_model, config.d_inner * 2, bias=config.bias)
        self.conv1d = nn.Conv1d(config.d_inner, config.d_inner, bias=config.conv_bias,
                                kernel_size=config.d_conv, groups=config.d_inner,
                                padding=config.d_conv - 1)
        self.activation = nn.SiLU()
        self.ssm = LinOSSSSM(config.d_inner, config.d_state, config.linoss_discretization,
                             config.a_init_method, config.dt_min, config.dt_max,
                             config.dt_init_floor, config.scan_algorithm)
        self.out_proj = nn.Linear(config.d_inner, config.d_model, bias=config.bias)

    def forward(self, x):
        L = x.shape[1]
        x, res = self.in_proj(x).split(self.config.d_inner, dim=-1)
        x = self.conv1d(x.transpose(-1, -2))[:, :, :L].transpose(-1, -2)
        x = self.ssm(self.activation(x))
        return self.out_proj(x * self.activation(res))


class LinOSSSSM(nn.Module):
    def __init__(self, d_inner: int, d_state: int, linoss_discretization: str,
                 a_init_method: str = "log_uniform", dt_min: float = 0.001, dt_max: float = 0.1,
                 dt_init_floor: float = 1e-4, scan_algorithm: str = "optimized"):
        super().__init__()
        self.d_inner = d_inner
        self.d_state = d_state
        self.linoss_discretization = linoss_discretization
        self.a_init_method = a_init_method
        self.dt_min, self.dt_max, self.dt_init_floor = dt_min, dt_max, dt_init_floor
        self.scan_algorithm = scan_algorithm
        self.dt_rank = math.ceil(d_inner / 16)
        self.x_proj = nn.Linear(d_inner, self.dt_rank + 4 * d_state, bias=False)
        self.dt_proj = nn.Linear(self.dt_rank, d_inner, bias=True)
        self.A_log = nn.Parameter(self._init_A_log())
        self.D = nn.Parameter(torch.randn(d_inner))
        self._init_projections()

    def _init_A_log(self):
        if self.a_init_method in ("log_uniform", "uniform"):
            return torch.rand(self.d_state) * 2.0
        if self.a_init_method == "relu":
            return torch.randn(self.d_state) * 0.1
        return torch.abs(torch.randn(self.d_state))

    def _init_projections(self):
        std = self.dt_rank ** -0.5
        nn.init.uniform_(self.dt_proj.weight, -std, std)
        lo, hi = math.log(self.dt_min), math.log(self.dt_max)
        dt = torch.exp(torch.rand(self.d_inner) * (hi - lo) + lo).clamp(min=self.dt_init_floor)
        with torch.no_grad():
            self.dt_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))
        nn.init.uniform_(self.x_proj.weight, -0.01, 0.01)

    def forward(self, x):
        P = self.d_state
        delta, Br, Bi, Cr, Ci = torch.split(self.x_proj(x), [self.dt_rank, P, P, P, P], dim=-1)
        delta = F.softplus(self.dt_proj(delta))
        A_diag = torch.exp(F.relu(self.A_log)) if self.a_init_method == "relu" else torch.exp(self.A_log)
        ys = apply_linoss_vectorized(self.linoss_discretization, A_diag, Br, Bi, Cr, Ci, x, delta,
                                     self.scan_algorithm)
        return ys + x * self.D

    def get_eigenspectrum_stats(self) -> Dict[str, torch.Tensor]:
        """Eigenvalue statistics of the transitions at a representative step 0.01."""
        with torch.no_grad():
            A = torch.exp(F.relu(self.A_log)) if self.a_init_method == "relu" else torch.exp(self.A_log)
            lam = 1.0 / torch.sqrt(1.0 + 0.01 ** 2 * torch.abs(A))
            return {"eigenval_min": A.min(), "eigenval_max": A.max(), "eigenval_mean": A.mean(),
                    "eigenval_std": A.std(), "lambda_mag_min": lam.min(),
                    "lambda_mag_max": lam.max(), "lambda_mag_mean": lam.mean(),
                    "A_log_min": self.A_log.min(), "A_log_max": self.A_log.max(),
                    "A_log_mean": self.A_log.mean()}


def parallel_scan_batched_complex(A_elements: torch.Tensor, b_elements: torch.Tensor
                                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Inclusive scan of (M, F) under (M_j M_i, M_j F_i + F_j): A (B, L, 4P) real,
    b (B, L, 2P) complex or real -> (A_scan, b_scan) (mamba_linoss.py:336-415)."""
    return scan2(A_elements, b_elements)


def parallel_scan_batched_complex_optimized(A_elements, b_elements):
    """Same result as parallel_scan_batched_complex (mamba_linoss.py:418-435)."""
    return scan2(A_elements, b_elements)


def apply_scan_vmap(M_elements, F_complex):
    """Same result as parallel_scan_batched_complex (mamba_linoss.py:680-699)."""
    return scan2(M_elements, F_complex)


def binary_operator_batched_complex(A_prev, b_prev, A_curr, b_curr):
    """(A_curr A_prev, A_curr b_prev + b_curr) on [A | B | C | D] blocks
    (mamba_linoss.py:561-605)."""
    return binary_operator_batched(A_prev, b_prev, A_curr, b_curr)


def apply_linoss_vectorized(discretization: str, A_diag: torch.Tensor, B_real_flat: torch.Tensor,
                            B_imag_flat: torch.Tensor, C_real_flat: torch.Tensor,
                            C_imag_flat: torch.Tensor, input_sequence: torch.Tensor,
                            delta: torch.Tensor, scan_algorithm: str = "optimized") -> torch.Tensor:
    """Selective LinOSS (mamba_linoss.py:608-677): delta averaged over channels,
    Bu = B * delta_bar, per-step IM / IMEX transitions, 2x2 scan, y = Re(sum_p C x2)
    broadcast over channels."""
    Bsz, L, ED = input_sequence.shape
    P = A_diag.shape[0]
    if discretization in ("IM", "IMEX"):
        # one fused kernel pair: transitions built per step in registers, output
        # contraction in the kernel (every scan_algorithm gives the correct scan)
        dbar = delta.float().mean(dim=-1)                                 # (B, L)
        y = linoss_selective(discretization, A_diag, dbar, B_real_flat, B_imag_flat,
                             C_real_flat, C_imag_flat)
        return y.unsqueeze(-1).expand(-1, -1, ED)
    Bc = torch.complex(B_real_flat.float(), B_imag_flat.float())
    Cc = torch.complex(C_real_flat.float(), C_imag_flat.float())
    dbar = delta.float().mean(dim=-1, keepdim=True)                       # (B, L, 1)
    Bu = Bc * dbar
    Ad = A_diag.float().view(1, 1, P)
    if discretization == "IM":
        S = 1.0 / (1.0 + dbar ** 2 * Ad)
        m11 = 1.0 - dbar ** 2 * Ad * S
        m12 = -dbar * Ad * S
        m21 = dbar * S
        m22 = S
        Fv = torch.cat([m11 * Bu, m21 * Bu], dim=-1)
    else:
        m11 = torch.ones(Bsz, L, P, device=delta.device)
        m12 = -dbar * Ad
        m21 = dbar.expand(Bsz, L, P)
        m22 = 1.0 - dbar ** 2 * Ad
        Fv = torch.cat([Bu, Bu * dbar], dim=-1)
    M = torch.cat([m11.expand(Bsz, L, P), m12, m21, m22.expand(Bsz, L, P)], dim=-1)
    _, X = scan2(M, Fv, want_mscan=False)
    out = torch.sum(Cc * X[:, :, P:], dim=-1).real
    return out.unsqueeze(-1).expand(-1, -1, ED)


def create_mamba_linoss_fast(d_model: int = 64, n_layer: int = 4) -> MambaLinOSS:
    return MambaLinOSS(MambaLinOSSConfig(d_model=d_model, n_layer=n_layer, scan_algorithm="vmap",
                                         use_vmap=True))


def create_mamba_linoss_balanced(d_model: int = 64, n_layer: int = 4) -> MambaLinOSS:
    return MambaLinOSS(MambaLinOSSConfig(d_model=d_model, n_layer=n_layer,
                                         scan_algorithm="optimized", use_vmap=False))


def create_mamba_linoss_memory_efficient(d_model: int = 64, n_layer: int = 4) -> MambaLinOSS:
    return MambaLinOSS(MambaLinOSSConfig(d_model=d_model, n_layer=n_layer, expand_factor=1,
                                         scan_algorithm="vectorized", use_vmap=False))
