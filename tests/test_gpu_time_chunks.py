"""The momentum selective scan split along time inside one GPU (time chunks
scanned by separate CTAs from carries folded out of per-chunk summaries),
against the fp64 oracle and against the same call unsplit.

Tolerance (stated for every comparison): max|gpu - ref| / max|ref| <= 1e-4 on
the output and on every gradient (fp32); bf16 activations 4e-3 against the
oracle run on the same bf16-rounded inputs.
"""
import numpy as np
import pytest
import torch

import oracle
from test_gpu_mmscan import assert_close, make_inputs, run_oracle

pytestmark = pytest.mark.gpu

TOL = 1e-4
TOL_BF16 = 4e-3
DEV = "cuda:0"


def run_chunked(inp, softplus, beta, alpha, time_chunk, dtype=torch.float32):
    from momentummamba_b200 import selective_scan_momentum_fn
    names = ["x", "delta", "A", "B", "C", "D", "z", "dbias"]
    act = {"x", "delta", "B", "C", "z"}
    ins = {}
    for k in names:
        v = inp[k]
        if v is None:
            ins[k] = None
            continue
        t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(DEV)
        if k in act:
            t = t.to(dtype)
        ins[k] = t.requires_grad_(True)
    y = selective_scan_momentum_fn(ins["x"], ins["delta"], ins["A"], ins["B"], ins["C"], ins["D"],
                                   z=ins["z"], delta_bias=ins["dbias"], delta_softplus=softplus,
                                   beta=beta, alpha=alpha, time_chunk=time_chunk)
    keys = [k for k in names if ins[k] is not None]
    dout = torch.from_numpy(np.ascontiguousarray(inp["dout"], dtype=np.float32)).to(DEV).to(dtype)
    grads = torch.autograd.grad(y, [ins[k] for k in keys], dout)
    torch.cuda.synchronize()
    return (y.detach().float().cpu().numpy(),
            {k: g.float().cpu().numpy() for k, g in zip(keys, grads)})


# (B, L, D, N, time_chunk): ragged lengths with forced chunks of 32-96 steps,
# a one-step last chunk, one chunk only (L <= chunk), and N = 8 / 32 / 64
CASES = [
    (1, 1, 16, 16, 32),
    (2, 33, 24, 16, 32),
    (1, 257, 64, 16, 64),
    (2, 300, 40, 16, 96),
    (1, 1000, 32, 16, 128),
    (3, 129, 16, 8, 32),
    (1, 200, 20, 32, 64),
    (1, 160, 16, 64, 32),
]


@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_forced_time_chunks_vs_oracle(case):
    Bsz, L, Dm, N, tc = case
    rng = np.random.default_rng(1000 + L + Dm)
    inp = make_inputs(rng, Bsz, L, Dm, N, z=True, bias=True, Dskip=True)
    y, g = run_chunked(inp, True, 0.9, 1.0, tc)
    yo, go = run_oracle(**inp, softplus=True, beta=0.9, alpha=1.0)
    assert_close(y, yo, "y", TOL)
    for k in go:
        assert_close(g[k], go[k], "d" + k, TOL)


def test_chunked_equals_unsplit_call():
    """Same inputs, the library's own split, forced chunks and no split."""
    rng = np.random.default_rng(7)
    inp = make_inputs(rng, 2, 1000, 64, 16, z=True, bias=True, Dskip=True)
    runs = {tc: run_chunked(inp, True, 0.6, 1.0, tc) for tc in (0, 64, -1)}
    y0, g0 = runs[-1]
    for tc in (0, 64):
        y, g = runs[tc]
        assert_close(y, y0, f"y chunk {tc}", TOL)
        for k in g0:
            assert_close(g[k], g0[k], f"d{k} chunk {tc}", TOL)


def test_automatic_split_long_sequence():
    """One sequence of 4096 steps x 64 channels: the library splits it on its own
    (8 one-warp CTAs would leave 140 SMs idle)."""
    from momentummamba_b200 import _lib
    lib = _lib.load()
    assert lib.mmb_mmscan_ckpt_floats(1, 4096, 64, 16) > 512 * 64 * 16 * 2
    rng = np.random.default_rng(11)
    inp = make_inputs(rng, 1, 4096, 64, 16, z=True, bias=True, Dskip=True)
    y, g = run_chunked(inp, True, 0.8, 1.0, 0)
    yo, go = run_oracle(**inp, softplus=True, beta=0.8, alpha=1.0)
    assert_close(y, yo, "y", TOL)
    for k in go:
        assert_close(g[k], go[k], "d" + k, TOL)


def test_forced_time_chunks_bf16():
    rng = np.random.default_rng(5)
    inp = make_inputs(rng, 2, 300, 64, 16, z=True, bias=True, Dskip=True)
    # the oracle sees the same bf16-rounded activations
    for k in ("x", "delta", "B", "C", "z", "dout"):
        inp[k] = torch.from_numpy(inp[k]).to(torch.bfloat16).double().numpy()
    y, g = run_chunked(inp, True, 0.9, 1.0, 64, dtype=torch.bfloat16)
    yo, go = run_oracle(**inp, softplus=True, beta=0.9, alpha=1.0)
    assert_close(y, yo, "y", TOL_BF16)
    for k in go:
        assert_close(g[k], go[k], "d" + k, TOL_BF16)
