"""B200-native (sm_100a) momentum selective scan and LinOSS 2x2 scan.

Drop-in modules mirroring the reference's entry points:
    momentummamba_b200.pscan                    pscan, PScan
    momentummamba_b200.momentum_scan_cuda       momentum_scan_cuda, MomentumScanCUDA
    momentummamba_b200.warp_momentum_scan_cuda  warp_momentum_scan_cuda
    momentummamba_b200.mamba_momentum           MambaMomentumConfig, MambaMomentum, ...
    momentummamba_b200.selective_scan           selective_scan_momentum_fn (fused op)
All compute runs in the in-tree C-ABI library libmomentum_scan_b200.so
(include/momentum_scan_b200.h); there is no CPU path.
"""
from .selective_scan import selective_scan_momentum_fn  # noqa: F401

__all__ = ["selective_scan_momentum_fn"]
