"""MambaMomentum on the sm_100a scan kernels -- drop-in for the reference's
mamba_momentum.py.

Same configuration dataclass, module tree and parameter names as the reference
(so its state_dicts load unchanged), same ``pscan_mode`` values
(mamba_momentum.py:64-68), plus ``"b200"``.  Every mode runs on this package's
CUDA kernels; there is no CPU path:

  "cuda_sequential" (default), "b200"
      the fused selective-scan kernel; inside ``MambaMomentumBlock.forward`` the
      delta softplus + bias (mamba_momentum.py:244-247) and the SiLU(z) gate
      (:227-229) run inside the same kernel.
  "pscan_sequential", "specialized"
      the reference's two-scan formulation (:325-368): materialised deltaA and
      alpha*deltaB*x, then v = pscan(beta, u), h = pscan(deltaA, v) on the
      PScan-layout kernel (one scan when |beta| < 1e-6).
  "sequential"
      the row-scan kernel of momentum_scan_cuda on the materialised tensors.

In every mode the block's causal depthwise conv1d + SiLU is one kernel
(conv.conv1d_silu, no transposes), and ``step()`` runs the conv-cache update
and the state update (with the dt softplus and the SiLU(z) gate) as one kernel
each (conv.conv1d_step, conv.mmscan_step).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from .conv import conv1d_silu, conv1d_step, mmscan_step
from .momentum_scan_cuda import momentum_scan_cuda
from .pscan import pscan
from .selective_scan import selective_scan_momentum_fn

CUDA_AVAILABLE = True  # the kernels are this package; they fail loudly if absent

_FUSED_MODES = ("cuda_sequential", "b200")


@dataclass
class MambaMomentumConfig:
    d_model: int
    n_layers: int
    dt_rank: Union[int, str] = "auto"
    d_state: int = 16
    expand_factor: int = 2
    d_conv: int = 4

    dt_min: float = 0.001
    dt_max: float = 0.1
    dt_init: str = "random"
    dt_scale: float = 1.0
    dt_init_floor = 1e-4

    momentum_beta: float = 0.6
    momentum_alpha: float = 1.0

    rms_norm_eps: float = 1e-5
    base_std: float = 0.02

    bias: bool = False
    conv_bias: bool = True
    inner_layernorms: bool = False

    mup: bool = False
    mup_base_width: float = 128

    pscan: bool = True
    pscan_mode: str = "cuda_sequential"

    def __post_init__(self):
        self.d_inner = self.expand_factor * self.d_model
        if self.dt_rank == "auto":
            self.dt_rank = math.ceil(self.d_model / 16)
        if self.mup:
            self.mup_width_mult = self.d_model / self.mup_base_width


class RMSNorm(nn.Module):
    def __init__(self, d_model: int, eps: float = 1e-5, use_mup: bool = False):
        super().__init__()
        self.use_mup = use_mup
        self.eps = eps
        if not use_mup:
            self.weight = nn.Parameter(torch.ones(d_model))

    def forward(self, x):
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)
        return y if self.use_mup else y * self.weight


class MambaMomentum(nn.Module):
    def __init__(self, config: MambaMomentumConfig):
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([ResidualBlock(config) for _ in range(config.n_layers)])

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return x

    def step(self, x, caches):
        for i, layer in enumerate(self.layers):
            x, caches[i] = layer.step(x, caches[i])
        return x, caches


class ResidualBlock(nn.Module):
    def __init__(self, config: MambaMomentumConfig):
        super().__init__()
        self.mixer = MambaMomentumBlock(config)
        self.norm = RMSNorm(config.d_model, config.rms_norm_eps, config.mup)

    def forward(self, x):
        return self.mixer(self.norm(x)) + x

    def step(self, x, cache):
        out, cache = self.mixer.step(self.norm(x), cache)
        return out + x, cache


class MambaMomentumBlock(nn.Module):
    def __init__(self, config: MambaMomentumConfig):
        super().__init__()
        self.config = config
        ed, n, r = config.d_inner, config.d_state, config.dt_rank
        self.in_proj = nn.Linear(config.d_model, 2 * ed, bias=config.bias)
        self.conv1d = nn.Conv1d(ed, ed, kernel_size=config.d_conv, bias=config.conv_bias,
                                groups=ed, padding=config.d_conv - 1)
        self.x_proj = nn.Linear(ed, r + 2 * n, bias=False)
        self.dt_proj = nn.Linear(r, ed, bias=True)

        # dt_proj init: uniform weight, bias = softplus^-1(dt), dt log-uniform in
        # [dt_min, dt_max] (the S4/Mamba recipe the reference follows)
        std = r ** -0.5 * config.dt_scale
        if config.dt_init == "constant":
            nn.init.constant_(self.dt_proj.weight, std)
        elif config.dt_init == "random":
            nn.init.uniform_(self.dt_proj.weight, -std, std)
        else:
            raise NotImplementedError
        lo, hi = math.log(config.dt_min), math.log(config.dt_max)
        dt = torch.exp(torch.rand(ed) * (hi - lo) + lo).clamp(min=config.dt_init_floor)
        with torch.no_grad():
            self.dt_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))

        # S4D-real A = -(1..N) per channel, stored as log
        self.A_log = nn.Parameter(torch.log(torch.arange(1, n + 1, dtype=torch.float32).repeat(ed, 1)))
        self.A_log._no_weight_decay = True
        self.D = nn.Parameter(torch.ones(ed))
        self.D._no_weight_decay = True

        self.momentum_beta = config.momentum_beta
        self.momentum_alpha = config.momentum_alpha
        self.out_proj = nn.Linear(ed, config.d_model, bias=config.bias)

        if config.inner_layernorms:
            self.dt_layernorm = RMSNorm(r, config.rms_norm_eps, config.mup)
            self.B_layernorm = RMSNorm(n, config.rms_norm_eps, config.mup)
            self.C_layernorm = RMSNorm(n, config.rms_norm_eps, config.mup)
        else:
            self.dt_layernorm = self.B_layernorm = self.C_layernorm = None

    def _apply_layernorms(self, dt, B, C):
        if self.dt_layernorm is not None:
            dt = self.dt_layernorm(dt)
        if self.B_layernorm is not None:
            B = self.B_layernorm(B)
        if self.C_layernorm is not None:
            C = self.C_layernorm(C)
        return dt, B, C

    # ------------------------------------------------------------------ #
    def _conv_silu(self, x):
        """silu(causal depthwise conv1d(x)) in one kernel (mamba_momentum.py:217-223)."""
        return conv1d_silu(x, self.conv1d.weight, self.conv1d.bias)

    def forward(self, x):
        xz = self.in_proj(x)
        x, z = xz.chunk(2, dim=-1)
        x = self._conv_silu(x)
        if self.config.pscan and self.config.pscan_mode in _FUSED_MODES:
            y = self._ssm_fused(x, z)
        else:
            y = self.ssm_momentum(x) * F.silu(z)
        return self.out_proj(y)

    def _project(self, x):
        A = -torch.exp(self.A_log.float())
        dbc = self.x_proj(x)
        r, n = self.config.dt_rank, self.config.d_state
        delta, B, C = torch.split(dbc, [r, n, n], dim=-1)
        delta, B, C = self._apply_layernorms(delta, B, C)
        return A, delta, B, C

    def _ssm_fused(self, x, z):
        """ssm_momentum + gate in one kernel: softplus(dt_proj(delta)) and y*silu(z) fused."""
        A, delta, B, C = self._project(x)
        delta_raw = F.linear(delta, self.dt_proj.weight)  # (B, L, ED), bias added in-kernel
        return selective_scan_momentum_fn(x, delta_raw, A, B, C, self.D.float(), z=z,
                                          delta_bias=self.dt_proj.bias.float(),
                                          delta_softplus=True, beta=self.momentum_beta,
                                          alpha=self.momentum_alpha)

    def ssm_momentum(self, x):
        A, delta, B, C = self._project(x)
        delta = F.softplus(F.linear(delta, self.dt_proj.weight, self.dt_proj.bias))
        return self.selective_scan_momentum(x, delta, A, B, C, self.D.float())

    def selective_scan_momentum(self, x, delta, A, B, C, D):
        """x, delta (B, L, ED); A (ED, N); B, C (B, L, N); D (ED) -> y (B, L, ED)."""
        mode = self.config.pscan_mode
        beta, alpha = self.momentum_beta, self.momentum_alpha
        if mode in _FUSED_MODES:
            return selective_scan_momentum_fn(x, delta, A, B, C, D, beta=beta, alpha=alpha)
        deltaA = torch.exp(delta.unsqueeze(-1) * A)                    # (B, L, ED, N)
        u = alpha * (delta.unsqueeze(-1) * B.unsqueeze(2)) * x.unsqueeze(-1)
        if mode == "sequential":
            h = self._sequential_momentum_scan(deltaA, beta, u)
        else:
            h = self._specialized_momentum_pscan(deltaA, beta, u)
        return (h @ C.unsqueeze(-1)).squeeze(3) + D * x

    def _specialized_momentum_pscan(self, deltaA, beta, momentum_input):
        """Two chained diagonal scans on (B, L, ED, N) (mamba_momentum.py:325-368)."""
        if abs(beta) < 1e-6:
            return pscan(deltaA, momentum_input)
        v = pscan(torch.full_like(deltaA, beta), momentum_input)
        return pscan(deltaA, v)

    def _cuda_momentum_scan_sequential(self, deltaA, beta, momentum_input,
                                       cuda_optimized_format=False):
        """Row scan on (B, ED, N, L) or, when not pre-formatted, (B, L, ED, N) tensors
        (mamba_momentum.py:370-413)."""
        if cuda_optimized_format:
            Bsz, ED, N, L = deltaA.shape
            h = momentum_scan_cuda(deltaA.reshape(-1, L), beta, momentum_input.reshape(-1, L))
            return h.view(Bsz, ED, N, L)
        Bsz, L, ED, N = deltaA.shape
        a = deltaA.permute(0, 2, 3, 1).reshape(-1, L)
        u = momentum_input.permute(0, 2, 3, 1).reshape(-1, L)
        return momentum_scan_cuda(a, beta, u).view(Bsz, ED, N, L).permute(0, 3, 1, 2)

    def _sequential_momentum_scan(self, deltaA, beta, momentum_input):
        """The plain recurrence on (B, L, ED, N) (mamba_momentum.py:415-435), on the row kernel."""
        return self._cuda_momentum_scan_sequential(deltaA, beta, momentum_input, False)

    # -------------------------- inference -------------------------- #
    def step(self, x, cache):
        """One token (mamba_momentum.py:439-471); cache = (h, v, conv inputs).
        The conv-cache update and the state update with the dt softplus and the
        SiLU(z) gate are one kernel each; the returned cache is new tensors, as
        in the reference."""
        h, v, inputs = cache
        xz = self.in_proj(x)
        x, z = xz.chunk(2, dim=1)
        x, inputs = conv1d_step(x, inputs, self.conv1d.weight, self.conv1d.bias)
        y, h, v = self._ssm_step(x, h, v, z)
        return self.out_proj(y), (h, v, inputs)

    def _ssm_step(self, x, h, v, z):
        A, delta, B, C = self._project(x)
        delta_raw = F.linear(delta, self.dt_proj.weight)  # bias and softplus in-kernel
        return mmscan_step(x, delta_raw, A, B, C, h, v, D=self.D.float(), z=z,
                           delta_bias=self.dt_proj.bias.float(), delta_softplus=True,
                           beta=self.momentum_beta, alpha=self.momentum_alpha)

    def ssm_momentum_step(self, x, h, v):
        """Single-step state update (mamba_momentum.py:473-515): (y, h, v)."""
        return self._ssm_step(x, h, v, None)
