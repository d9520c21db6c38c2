"""The sequence-sharded scan protocol (momentummamba_b200.seqshard) on gloo
ranks over CPU: every rank scans its own time segment, the segment summaries
are all-gathered, the carries folded, and the parameter gradients all-reduced.

The per-segment operations here are the CPU oracle's (segment summary,
forward from a state, backward from an adjoint carry) and a numpy statement
of the two carry folds; the CUDA kernels behind the same operations are
checked against the oracle on the GPU.  The result on every rank must be its
segment of the whole-sequence scan, within fp64 round-off.
"""
import os
import socket
import types

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

BETA, ALPHA = 0.8, 1.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(L, seed=3, Bsz=2, Dm=8, N=16):
    rng = np.random.default_rng(seed)
    return dict(
        x=rng.standard_normal((Bsz, L, Dm)),
        delta=0.5 * rng.standard_normal((Bsz, L, Dm)) - 2.0,
        A=-np.tile(np.arange(1, N + 1, dtype=np.float64), (Dm, 1)) * rng.uniform(0.5, 1.5, (Dm, N)),
        B=rng.standard_normal((Bsz, L, N)), C=rng.standard_normal((Bsz, L, N)),
        D=rng.standard_normal(Dm), z=rng.standard_normal((Bsz, L, Dm)),
        bias=0.1 * rng.standard_normal(Dm), dout=rng.standard_normal((Bsz, L, Dm)))


class OracleOps:
    """Per-segment operations of the protocol on the fp64 CPU oracle."""

    @staticmethod
    def make_call(x, delta, A, B, C, D, z, delta_bias, softplus, beta, alpha):
        n = lambda t: None if t is None else t.detach().double().numpy()
        return types.SimpleNamespace(x=n(x), delta=n(delta), A=n(A), B=n(B), C=n(C), D=n(D),
                                     z=n(z), bias=n(delta_bias), softplus=softplus, beta=beta,
                                     alpha=alpha)

    @staticmethod
    def fwd_summary(c):
        import oracle
        return torch.from_numpy(oracle.mmscan_fwd_summary(c.x, c.delta, c.A, c.B, c.bias, c.softplus,
                                                          c.beta, c.alpha))

    @staticmethod
    def forward(c, state_in, need_ckpt):
        import oracle
        s = None if state_in is None else state_in.numpy()
        y = oracle.mmscan_fwd(c.x, c.delta, c.A, c.B, c.C, c.D, c.z, c.bias, c.softplus, c.beta,
                              c.alpha, state_in=s)
        return torch.from_numpy(y), s   # the "checkpoint" is the incoming state

    @staticmethod
    def bwd_summary(c, dout):
        import oracle
        r = oracle.mmscan_bwd(c.x, c.delta, c.A, c.B, c.C, c.D, c.z, c.bias, c.softplus, c.beta,
                              c.alpha, dout.double().numpy(), return_gstate=True)
        return torch.from_numpy(r[8])

    @staticmethod
    def backward(c, ckpt, dout, gstate_in):
        import oracle
        g = None if gstate_in is None else gstate_in.numpy()
        r = oracle.mmscan_bwd(c.x, c.delta, c.A, c.B, c.C, c.D, c.z, c.bias, c.softplus, c.beta,
                              c.alpha, dout.double().numpy(), state_in=ckpt, gstate_in=g)
        return tuple(None if t is None else torch.from_numpy(t) for t in r)

    @staticmethod
    def carry_fwd(summ, seg, seg_lens, beta):
        s = summ.numpy()
        h = np.zeros_like(s[0, :, :, 0])
        v = np.zeros_like(h)
        for j in range(seg):
            h, v = s[j, :, :, 2] * h + beta * s[j, :, :, 3] * v + s[j, :, :, 0], \
                beta ** seg_lens[j] * v + s[j, :, :, 1]
        return torch.from_numpy(np.stack([h, v], axis=2))

    @staticmethod
    def carry_bwd(summ, gsumm, seg, seg_lens, beta):
        s, g = summ.numpy(), gsumm.numpy()
        lam = np.zeros_like(s[0, :, :, 0])
        mu = np.zeros_like(lam)
        for j in range(len(seg_lens) - 1, seg, -1):
            lam, mu = s[j, :, :, 2] * lam + g[j, :, :, 0], \
                s[j, :, :, 3] * lam + beta ** seg_lens[j] * mu + g[j, :, :, 1]
        return torch.from_numpy(np.stack([lam, mu], axis=2))


def _worker(rank, world, port, seg_lens, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from momentummamba_b200.seqshard import seq_sharded_selective_scan
        L = sum(seg_lens)
        g = _inputs(L)
        a, b = sum(seg_lens[:rank]), sum(seg_lens[: rank + 1])
        seg = lambda k: torch.from_numpy(np.ascontiguousarray(g[k][:, a:b])).requires_grad_()
        x, delta, B, C, z = (seg(k) for k in ("x", "delta", "B", "C", "z"))
        A, D, bias = (torch.from_numpy(g[k]).requires_grad_() for k in ("A", "D", "bias"))
        y = seq_sharded_selective_scan(x, delta, A, B, C, D, z, bias, True, BETA, ALPHA,
                                       seg_lens=seg_lens, ops=OracleOps)
        y.backward(torch.from_numpy(np.ascontiguousarray(g["dout"][:, a:b])))
        grads = {k: t.grad.numpy() for k, t in
                 dict(x=x, delta=delta, A=A, B=B, C=C, D=D, z=z, bias=bias).items()}
        q.put((rank, y.detach().numpy(), grads))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("seg_lens", [(48, 53), (40, 16, 37)])
def test_sequence_sharded_protocol_matches_the_whole_sequence(seg_lens):
    import oracle
    world, port = len(seg_lens), _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, list(seg_lens), q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=180) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = _inputs(sum(seg_lens))
    y = oracle.mmscan_fwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], g["bias"],
                          True, BETA, ALPHA)
    full = oracle.mmscan_bwd(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], g["bias"],
                             True, BETA, ALPHA, g["dout"])
    rel = lambda a, b: float(np.abs(a - b).max() / np.abs(b).max())
    assert rel(np.concatenate([r[1] for r in res], 1), y) < 1e-10
    names = ["x", "delta", "A", "B", "C", "D", "z", "bias"]
    idx = dict(x=0, delta=1, A=2, B=3, C=4, D=5, z=6, bias=7)
    for k in names:
        want = full[idx[k]]
        if k in ("A", "D", "bias"):
            for r in res:                      # all-reduced: the full sum on every rank
                assert rel(r[2][k], want) < 1e-10, k
        else:
            got = np.concatenate([r[2][k] for r in res], 1)
            assert rel(got, want) < 1e-10, k


class _InjectedFault(RuntimeError):
    pass


def _faulty_worker(rank, world, port, seg_lens, fail_rank, q):
    """One rank of the protocol whose rank `fail_rank` raises between the forward
    all-gather and the carry fold, then leaves without another collective."""
    import datetime
    import time
    import torch.distributed as dist

    class FaultyOps(OracleOps):
        @staticmethod
        def carry_fwd(summ, seg, lens, beta):
            if seg == fail_rank:
                raise _InjectedFault(f"rank {seg}: injected failure before the fold")
            return OracleOps.carry_fwd(summ, seg, lens, beta)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    t0 = time.monotonic()
    outcome = "finished"
    try:
        from momentummamba_b200.seqshard import seq_sharded_selective_scan
        L = sum(seg_lens)
        g = _inputs(L)
        a, b = sum(seg_lens[:rank]), sum(seg_lens[: rank + 1])
        seg = lambda k: torch.from_numpy(np.ascontiguousarray(g[k][:, a:b])).requires_grad_()
        x, delta, B, C, z = (seg(k) for k in ("x", "delta", "B", "C", "z"))
        A, D, bias = (torch.from_numpy(g[k]).requires_grad_() for k in ("A", "D", "bias"))
        y = seq_sharded_selective_scan(x, delta, A, B, C, D, z, bias, True, BETA, ALPHA,
                                       seg_lens=seg_lens, ops=FaultyOps)
        y.backward(torch.from_numpy(np.ascontiguousarray(g["dout"][:, a:b])))
    except _InjectedFault:
        outcome = "injected"
    except Exception as e:  # the survivors: the next collective must fail, not hang
        outcome = f"error: {type(e).__name__}"
    q.put((rank, outcome, time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)  # leave without destroy_process_group: a rank that died


@pytest.mark.parametrize("seg_lens,fail_rank", [((48, 53), 1), ((40, 16, 37), 1)])
def test_a_failing_rank_ends_the_others_collectives_with_an_error(seg_lens, fail_rank):
    """A rank that raises between the forward all-gather and the fold and then
    leaves: every other rank gets an error from its next collective within the
    process-group timeout (10 s) instead of waiting for good."""
    world, port = len(seg_lens), _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_faulty_worker,
                         args=(r, world, port, list(seg_lens), fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=120) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, outcome, secs in res:
        if rank == fail_rank:
            assert outcome == "injected"
        else:
            assert outcome.startswith("error"), (rank, outcome)
            assert secs < 60.0, (rank, secs)
