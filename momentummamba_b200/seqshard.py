"""Momentum selective scan over a sequence split along time across ranks.

Each rank of a process group holds one contiguous time segment of every
sequence (rank r the r-th segment) and calls
``seq_sharded_selective_scan`` with it; the result on each rank is that
segment of the scan of the whole sequence, and the gradients are those of the
whole-sequence scan (the parameter gradients dA, dD, d(delta_bias) summed over
all segments on every rank).  The reference scans a sequence on one device
only; this is the long-sequence extension of its scan (mamba_momentum.py:256-323).

Protocol (no peer memory access: remote data only ever arrives through NCCL
into local memory):

forward
  1. summary of the local segment from a zero state:
     [h^0 | v^0 | P | Q'] per (b, d, n)                      (mmb_mmscan_fwd_summary)
  2. all-gather of the summaries                              (NCCL all_gather)
  3. fold of the segments before this one into its incoming state
                                                              (mmb_mmscan_carry_fwd)
  4. the scan of the segment from that state, with checkpoints (mmb_mmscan_forward)
backward
  1. adjoint summary [lam^0 | mu^0] of the segment            (mmb_mmscan_bwd_summary)
  2. all-gather of the adjoint summaries                      (NCCL all_gather)
  3. fold of the segments after this one (with their P, Q') into the incoming
     adjoint pair                                             (mmb_mmscan_carry_bwd)
  4. the backward of the segment from it                      (mmb_mmscan_backward)
  5. all-reduce (sum) of dA, dD, d(delta_bias)                (NCCL all_reduce)

Every segment but the last must have a length that is a multiple of 8 (the
adjoint pair enters a segment at the end of an 8-step window).

The per-segment operations are those of ``SegmentOps`` (the CUDA kernels);
the orchestration takes any object with the same methods, which is how the
CPU tests drive the protocol over gloo with the oracle in its place.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib
from .selective_scan import ScanCall


class SegmentOps:
    """The per-segment operations on the CUDA kernels."""

    @staticmethod
    def make_call(x, delta, A, B, C, D, z, delta_bias, softplus, beta, alpha):
        return ScanCall(x, delta, A, B, C, D, z, delta_bias, softplus, beta, alpha)

    @staticmethod
    def fwd_summary(call):
        return call.fwd_summary()

    @staticmethod
    def forward(call, state_in, need_ckpt):
        out, ckpt, _ = call.forward(need_ckpt, state_in=state_in)
        return out, ckpt

    @staticmethod
    def bwd_summary(call, dout):
        return call.bwd_summary(dout)

    @staticmethod
    def backward(call, ckpt, dout, gstate_in):
        return call.backward(ckpt, dout, gstate_in=gstate_in)[:8]

    @staticmethod
    def carry_fwd(summaries, seg, seg_lens, beta):
        nseg, Bsz, Dm, _, N = summaries.shape
        state = torch.empty((Bsz, Dm, 2, N), device=summaries.device)
        lens = (ctypes.c_int64 * nseg)(*seg_lens)
        with torch.cuda.device(summaries.device):
            st = _lib.load().mmb_mmscan_carry_fwd(nseg, seg, lens, Bsz, Dm, N, float(beta),
                                                  _lib.ptr(summaries), _lib.ptr(state),
                                                  _lib.stream_of(summaries))
        _lib.check(st, "mmb_mmscan_carry_fwd")
        return state

    @staticmethod
    def carry_bwd(summaries, gsummaries, seg, seg_lens, beta):
        nseg, Bsz, Dm, _, N = summaries.shape
        gstate = torch.empty((Bsz, Dm, 2, N), device=summaries.device)
        lens = (ctypes.c_int64 * nseg)(*seg_lens)
        with torch.cuda.device(summaries.device):
            st = _lib.load().mmb_mmscan_carry_bwd(nseg, seg, lens, Bsz, Dm, N, float(beta),
                                                  _lib.ptr(summaries), _lib.ptr(gsummaries),
                                                  _lib.ptr(gstate), _lib.stream_of(summaries))
        _lib.check(st, "mmb_mmscan_carry_bwd")
        return gstate


def _gather(t: torch.Tensor, group) -> torch.Tensor:
    """(world, *t.shape): every rank's t in rank order."""
    world = dist.get_world_size(group)
    out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out.view((world,) + tuple(t.shape))


class SeqShardedScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, delta, A, B, C, D, z, delta_bias, softplus, beta, alpha, group, seg_lens,
                ops):
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        call = ops.make_call(x, delta, A, B, C, D, z, delta_bias, softplus, beta, alpha)
        summaries = _gather(ops.fwd_summary(call), group)
        state_in = ops.carry_fwd(summaries, rank, seg_lens, beta) if rank > 0 else None
        need_grad = any(ctx.needs_input_grad[:8])
        out, ckpt = ops.forward(call, state_in, need_grad)
        ctx.call, ctx.ckpt, ctx.summaries = call, ckpt, summaries
        ctx.cfg = (group, list(seg_lens), float(beta), rank, world, ops)
        ctx.in_dtypes = [None if t is None else t.dtype
                         for t in (x, delta, A, B, C, D, z, delta_bias)]
        return out

    @staticmethod
    def backward(ctx, dout):
        group, seg_lens, beta, rank, world, ops = ctx.cfg
        call = ctx.call
        # rank 0's adjoint summary feeds no fold; it still joins the all-gather
        gs = ops.bwd_summary(call, dout) if rank > 0 else None
        if gs is None:
            Bsz, _, Dm = dout.shape
            gs = torch.zeros((Bsz, Dm, 2, ctx.summaries.shape[-1]), device=dout.device,
                             dtype=ctx.summaries.dtype)
        gsummaries = _gather(gs, group)
        gstate_in = (ops.carry_bwd(ctx.summaries, gsummaries, rank, seg_lens, beta)
                     if rank < world - 1 else None)
        dx, ddelta, dA, dB, dC, dD, dz, ddb = ops.backward(call, ctx.ckpt, dout, gstate_in)
        # parameter gradients: sums over every segment
        parts = [dA.reshape(-1)] + [g for g in (dD, ddb) if g is not None]
        flat = torch.cat(parts)
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        dA = flat[: dA.numel()].view_as(dA)
        off = dA.numel()
        if dD is not None:
            dD = flat[off: off + dD.numel()]
            off += dD.numel()
        if ddb is not None:
            ddb = flat[off: off + ddb.numel()]
        res = []
        for need, g, dt in zip(ctx.needs_input_grad[:8], (dx, ddelta, dA, dB, dC, dD, dz, ddb),
                               ctx.in_dtypes):
            res.append((g if dt is None or g.dtype == dt else g.to(dt)) if need and g is not None
                       else None)
        ctx.call = ctx.ckpt = ctx.summaries = None
        return (*res,) + (None,) * 6


def seq_sharded_selective_scan(x, delta, A, B, C, D=None, z=None, delta_bias=None,
                               delta_softplus=False, beta=0.6, alpha=1.0, group=None,
                               seg_lens: Optional[Sequence[int]] = None, ops=SegmentOps):
    """Momentum selective scan of a sequence split along time over ``group``.

    x, delta, z, B, C hold this rank's segment (batch, seg_len, ...); A, D,
    delta_bias are the shared parameters.  ``seg_lens`` lists every rank's
    segment length in rank order (default: all equal to this rank's).  Every
    length but the last must be a multiple of 8."""
    world = dist.get_world_size(group)
    L = x.shape[1]
    seg_lens = [L] * world if seg_lens is None else [int(s) for s in seg_lens]
    rank = dist.get_rank(group)
    if len(seg_lens) != world or seg_lens[rank] != L:
        raise ValueError("seg_lens must list every rank's segment length (this rank's = x.shape[1])")
    if any(s % 8 for s in seg_lens[:-1]):
        raise ValueError("every segment but the last needs a length that is a multiple of 8")
    if world > 64:
        raise ValueError("at most 64 segments")
    return SeqShardedScanFn.apply(x, delta, A, B, C, D, z, delta_bias, bool(delta_softplus),
                                  float(beta), float(alpha), group, tuple(seg_lens), ops)
