"""GPU parity of the segment entry points (state carries, segment summaries,
carry folds) and of bf16 activations, against the fp64 CPU oracle.

A sequence split into segments and scanned segment by segment through
mmb_mmscan_fwd_summary -> mmb_mmscan_carry_fwd -> mmb_mmscan_forward (and the
adjoint mirror for the backward) must reproduce the scan of the whole
sequence.  Here the segments run one after another on one GPU; the
multi-GPU path runs the same calls with an all-gather in between.

Tolerances (max|gpu - ref| / max|ref|):
  fp32 activations: 1e-4 on every output and gradient;
  bf16 activations: 4e-3 on the bf16 outputs (out, dx, ddelta, dz; bf16
  rounding alone is up to 2^-9 = 2e-3 of the largest value) and 1e-4 on the
  fp32 ones (dA, dB, dC, dD, d(delta_bias)), the oracle running in fp64 on the
  same bf16-rounded inputs.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 1e-4
TOL_BF16 = 4e-3
BETA, ALPHA = 0.8, 1.0


def rel(a, b):
    a = a.detach().double().cpu().numpy() if isinstance(a, torch.Tensor) else a
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def make(seed, Bsz, L, Dm, N, gate=True, bias=True):
    rng = np.random.default_rng(seed)
    g = dict(x=rng.standard_normal((Bsz, L, Dm)),
             delta=0.5 * rng.standard_normal((Bsz, L, Dm)) - 2.0,
             A=-np.tile(np.arange(1, N + 1, dtype=np.float64), (Dm, 1)) * rng.uniform(0.5, 1.5, (Dm, N)),
             B=rng.standard_normal((Bsz, L, N)), C=rng.standard_normal((Bsz, L, N)),
             D=rng.standard_normal(Dm), z=rng.standard_normal((Bsz, L, Dm)) if gate else None,
             bias=0.1 * rng.standard_normal(Dm) if bias else None,
             dout=rng.standard_normal((Bsz, L, Dm)))
    return g


def to_dev(g, dtype):
    act = ("x", "delta", "B", "C", "z", "dout")
    return {k: None if v is None else
            torch.from_numpy(np.ascontiguousarray(v)).to(DEV, dtype if k in act else torch.float32)
            for k, v in g.items()}


def rounded(t):
    """the values the kernels see, as fp64 numpy (bf16-rounded where bf16)"""
    return {k: None if v is None else v.double().cpu().numpy() for k, v in t.items()}


def call_for(t, a, b, softplus=True):
    from momentummamba_b200.selective_scan import ScanCall
    s = lambda k: None if t[k] is None else t[k][:, a:b]
    return ScanCall(s("x"), s("delta"), t["A"], s("B"), s("C"), t["D"], s("z"), t["bias"],
                    softplus, BETA, ALPHA)


def run_segments(t, seg_lens, softplus=True):
    """forward and backward of the whole sequence, one segment at a time"""
    from momentummamba_b200.seqshard import SegmentOps as ops
    edges = np.cumsum([0] + list(seg_lens))
    calls = [call_for(t, a, b, softplus) for a, b in zip(edges[:-1], edges[1:])]
    summ = torch.stack([c.fwd_summary() for c in calls])
    outs, ckpts = [], []
    for j, c in enumerate(calls):
        st = ops.carry_fwd(summ, j, seg_lens, BETA) if j > 0 else None
        y, ck = ops.forward(c, st, True)
        outs.append(y)
        ckpts.append(ck)
    douts = [t["dout"][:, a:b] for a, b in zip(edges[:-1], edges[1:])]
    gsumm = torch.stack([c.bwd_summary(d) for c, d in zip(calls, douts)])
    grads = []
    for j, c in enumerate(calls):
        gi = ops.carry_bwd(summ, gsumm, j, seg_lens, BETA) if j < len(calls) - 1 else None
        grads.append(ops.backward(c, ckpts[j], douts[j], gi))
    torch.cuda.synchronize()
    y = torch.cat(outs, 1)
    cat = lambda i: torch.cat([g[i] for g in grads], 1)
    tot = lambda i: None if grads[0][i] is None else sum(g[i] for g in grads)
    return y, dict(x=cat(0), delta=cat(1), A=tot(2), B=cat(3), C=cat(4), D=tot(5),
                   z=None if grads[0][6] is None else cat(6), bias=tot(7))


def oracle_full(r, softplus=True):
    y = oracle.mmscan_fwd(r["x"], r["delta"], r["A"], r["B"], r["C"], r["D"], r["z"], r["bias"],
                          softplus, BETA, ALPHA)
    g = oracle.mmscan_bwd(r["x"], r["delta"], r["A"], r["B"], r["C"], r["D"], r["z"], r["bias"],
                          softplus, BETA, ALPHA, r["dout"])
    return y, dict(zip(["x", "delta", "A", "B", "C", "D", "z", "bias"], g))


FP32_OUT = ("A", "B", "C", "D", "bias")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("Bsz,Dm,N,seg_lens,gate", [
    (2, 64, 16, (64, 96, 45), True),      # 2 states per thread; ragged last segment
    (4, 512, 16, (256, 128, 256), True),  # 4 states per thread
    (2, 64, 64, (40, 8, 33), False),      # d_state 64, one-window segment
    (3, 256, 8, (104, 200), True),
])
def test_segments_reproduce_the_whole_sequence(dtype, Bsz, Dm, N, seg_lens, gate):
    t = to_dev(make(N + len(seg_lens), Bsz, sum(seg_lens), Dm, N, gate=gate), dtype)
    y, grads = run_segments(t, seg_lens)
    yo, go = oracle_full(rounded(t))
    lo = TOL_BF16 if dtype == torch.bfloat16 else TOL
    assert y.dtype == dtype
    assert rel(y, yo) <= lo, f"y {rel(y, yo):.2e}"
    for k, want in go.items():
        if want is None:
            continue
        tol = TOL if k in FP32_OUT else lo
        assert rel(grads[k], want) <= tol, f"d{k}: {rel(grads[k], want):.2e}"


@pytest.mark.parametrize("L", [45, 64, 1])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("Bsz,Dm", [(2, 64), (64, 256)])  # one- and two-channel kernels
def test_summaries_and_state_outputs(L, dtype, Bsz, Dm):
    """Summaries, state_out and gstate_out of one segment, including a ragged
    length whose last 8-step block runs past the end."""
    t = to_dev(make(7, Bsz, L, Dm, 16), dtype)
    r = rounded(t)
    c = call_for(t, 0, L)
    summ = c.fwd_summary()
    so = oracle.mmscan_fwd_summary(r["x"], r["delta"], r["A"], r["B"], r["bias"], True, BETA, ALPHA)
    assert rel(summ, so) <= TOL
    rng = np.random.default_rng(1)
    s_in = torch.from_numpy(rng.standard_normal((Bsz, Dm, 2, 16))).float().to(DEV)
    y, ck, s_out = c.forward(True, state_in=s_in, want_state=True)
    yo, s_outo = oracle.mmscan_fwd(r["x"], r["delta"], r["A"], r["B"], r["C"], r["D"], r["z"],
                                   r["bias"], True, BETA, ALPHA, state_in=s_in.double().cpu().numpy(),
                                   return_state=True)
    assert rel(y, yo) <= (TOL_BF16 if dtype == torch.bfloat16 else TOL)
    assert rel(s_out, s_outo) <= TOL
    gs = c.bwd_summary(t["dout"])
    go = oracle.mmscan_bwd(r["x"], r["delta"], r["A"], r["B"], r["C"], r["D"], r["z"], r["bias"],
                           True, BETA, ALPHA, r["dout"], return_gstate=True)[8]
    assert rel(gs, go) <= TOL
    # the full backward's outgoing pair, with and without an incoming one
    g_in = (torch.from_numpy(rng.standard_normal((Bsz, Dm, 2, 16))).float().to(DEV)
            if L % 8 == 0 else None)
    res = c.backward(ck, t["dout"], gstate_in=g_in, want_gstate=True)
    ro = oracle.mmscan_bwd(r["x"], r["delta"], r["A"], r["B"], r["C"], r["D"], r["z"], r["bias"],
                           True, BETA, ALPHA, r["dout"], state_in=s_in.double().cpu().numpy(),
                           gstate_in=None if g_in is None else g_in.double().cpu().numpy(),
                           return_gstate=True)
    assert rel(res[8], ro[8]) <= TOL
    assert rel(res[3], ro[3]) <= TOL                      # dB (fp32)
    assert rel(res[0], ro[0]) <= (TOL_BF16 if dtype == torch.bfloat16 else TOL)


def test_incoming_adjoint_needs_whole_windows():
    from momentummamba_b200 import _lib
    t = to_dev(make(2, 1, 12, 64, 16), torch.float32)
    c = call_for(t, 0, 12)
    _, ck, _ = c.forward(True)
    g_in = torch.zeros((1, 64, 2, 16), device=DEV)
    with pytest.raises(RuntimeError, match="status 2"):
        c.backward(ck, t["dout"], gstate_in=g_in)


def test_bf16_autograd_drop_in():
    """selective_scan_momentum_fn with bf16 activations: bf16 out and activation
    gradients, parameter gradients in the parameters' dtype."""
    from momentummamba_b200 import selective_scan_momentum_fn
    t = to_dev(make(5, 2, 200, 128, 16), torch.bfloat16)
    ins = {k: (v.clone().requires_grad_() if v is not None and k != "dout" else v) for k, v in t.items()}
    y = selective_scan_momentum_fn(ins["x"], ins["delta"], ins["A"], ins["B"], ins["C"], ins["D"],
                                   z=ins["z"], delta_bias=ins["bias"], delta_softplus=True,
                                   beta=BETA, alpha=ALPHA)
    keys = ["x", "delta", "A", "B", "C", "D", "z", "bias"]
    grads = torch.autograd.grad(y, [ins[k] for k in keys], t["dout"])
    assert y.dtype == torch.bfloat16
    for k, gr in zip(keys, grads):
        assert gr.dtype == ins[k].dtype, k
    yo, go = oracle_full(rounded(t))
    assert rel(y, yo) <= TOL_BF16
    for k, gr in zip(keys, grads):
        # dB, dC come back in bf16 (the dtype of B, C): bf16 rounding bound
        tol = TOL if k in ("A", "D", "bias") else TOL_BF16
        assert rel(gr, go[k]) <= tol, f"d{k}: {rel(gr, go[k]):.2e}"
