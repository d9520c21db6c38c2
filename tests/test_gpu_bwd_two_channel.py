"""The two-channel momentum backward (mmscan_bwd2_kernel: each thread owns 4
states of two channels, windows replayed in halves) against the fp64 oracle.

The library picks it for one-warp grids of at least 6 CTAs per SM, so the
shapes here are wide enough (B x ceil(D / channels per CTA) >= 888) while the
sequences stay short for the oracle.  Ragged channel counts leave the second
channel of some pairs outside D.

Tolerance (stated for every comparison): max|gpu - ref| / max|ref| <= 1e-4 on
the output and on every gradient (fp32); bf16 activations 4e-3 against the
oracle run on the same bf16-rounded inputs.
"""
import numpy as np
import pytest
import torch

from test_gpu_mmscan import assert_close, make_inputs, run_oracle
from test_gpu_time_chunks import run_chunked

pytestmark = pytest.mark.gpu

TOL = 1e-4
TOL_BF16 = 4e-3

# (B, L, D, N, z, softplus + bias, D skip, beta, time_chunk); channels per
# CTA: 32 (N = 8), 16 (N = 16), 8 (N = 32)
CASES = [
    (72, 37, 200, 16, True, True, True, 0.9, 0),     # D = 200: pairs 192-199 | 200-207
    (72, 40, 208, 16, False, False, True, 0.6, 0),   # no gate, no softplus
    (240, 19, 120, 8, True, True, False, 0.5, 0),    # N = 8, no D skip
    (64, 33, 140, 32, True, False, True, 0.7, 0),    # N = 32, D = 140 (half a CTA)
    (8, 1000, 200, 16, True, True, True, 0.9, 64),   # 16 forced time chunks
    (32, 300, 136, 16, True, True, True, 0.0, 96),   # beta = 0, ragged last chunk
]


@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_two_channel_backward_vs_oracle(case):
    Bsz, L, Dm, N, z, sp, Dskip, beta, tc = case
    rng = np.random.default_rng(Bsz * 1000 + L + Dm + N)
    inp = make_inputs(rng, Bsz, L, Dm, N, z=z, bias=sp, Dskip=Dskip)
    y, g = run_chunked(inp, sp, beta, 1.0, tc)
    yo, go = run_oracle(**inp, softplus=sp, beta=beta, alpha=1.0)
    assert_close(y, yo, "y", TOL)
    for k in go:
        assert_close(g[k], go[k], "d" + k, TOL)


def test_two_channel_backward_bf16():
    rng = np.random.default_rng(17)
    inp = make_inputs(rng, 72, 50, 200, 16, z=True, bias=True, Dskip=True)
    for k in ("x", "delta", "B", "C", "z", "dout"):
        inp[k] = torch.from_numpy(inp[k]).to(torch.bfloat16).double().numpy()
    y, g = run_chunked(inp, True, 0.9, 1.0, 0, dtype=torch.bfloat16)
    yo, go = run_oracle(**inp, softplus=True, beta=0.9, alpha=1.0)
    assert_close(y, yo, "y", TOL_BF16)
    for k in go:
        assert_close(g[k], go[k], "d" + k, TOL_BF16)


def _bwd_kernels(Bsz, L, Dm, N):
    """Names of the scan kernels one backward call of this shape launches."""
    from momentummamba_b200 import selective_scan_momentum_fn
    dev = "cuda:0"
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(Bsz, L, Dm, device=dev, generator=g, requires_grad=True)
    delta = torch.rand(Bsz, L, Dm, device=dev, generator=g)
    A = -torch.rand(Dm, N, device=dev, generator=g) - 0.5
    B = torch.randn(Bsz, L, N, device=dev, generator=g)
    C = torch.randn(Bsz, L, N, device=dev, generator=g)
    y = selective_scan_momentum_fn(x, delta, A, B, C, None)
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA],
                                acc_events=True) as prof:
        y.backward(torch.ones_like(y))
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if "mmscan_bwd" in e.name]


def test_dispatch_by_grid_size():
    """Wide grids run the two-channel kernel, narrow ones the one-channel kernel."""
    wide = _bwd_kernels(64, 16, 512, 16)    # 2048 two-channel CTAs
    narrow = _bwd_kernels(4, 16, 256, 16)   # 64
    assert any("mmscan_bwd2_kernel" in n for n in wide), wide
    assert not any("mmscan_bwd2_kernel" in n for n in narrow), narrow
    assert any("mmscan_bwd_kernel" in n for n in narrow), narrow
