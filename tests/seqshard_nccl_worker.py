"""Worker for test_gpu_seqshard_nccl.py, run under torch.distributed.run with
one rank per GPU: the sequence-sharded scan over NCCL against the unsplit scan
on one GPU (itself checked against the CPU oracle by the other GPU tests).

Every rank builds the same whole-sequence inputs, scans them alone, then scans
its own segment through seq_sharded_selective_scan and compares its segment of
the output and gradients (and the all-reduced parameter gradients).
Exit status 0 on agreement (max|a - b| / max|b| <= 1e-4 fp32, 4e-3 bf16 outputs).
"""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from momentummamba_b200 import selective_scan_momentum_fn  # noqa: E402
from momentummamba_b200.seqshard import seq_sharded_selective_scan  # noqa: E402


def rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max())


def run(dtype, rank, world, dev):
    seg_lens = [256] * (world - 1) + [203]       # ragged last segment
    L, Bsz, D, N = sum(seg_lens), 2, 256, 16
    g = torch.Generator(device=dev).manual_seed(11)
    mk = lambda *s: torch.randn(*s, device=dev, generator=g)
    x, z, dout = mk(Bsz, L, D).to(dtype), mk(Bsz, L, D).to(dtype), mk(Bsz, L, D).to(dtype)
    delta = (0.5 * mk(Bsz, L, D) - 2.0).to(dtype)
    Bm, Cm = mk(Bsz, L, N).to(dtype), mk(Bsz, L, N).to(dtype)
    A = -torch.arange(1, N + 1, device=dev, dtype=torch.float32).repeat(D, 1) * (
        0.5 + torch.rand(D, 1, device=dev, generator=g))
    Dk, bias = mk(D), 0.1 * mk(D)
    kw = dict(delta_softplus=True, beta=0.8, alpha=1.0)
    full = [t.clone().requires_grad_() for t in (x, delta, A, Bm, Cm, Dk, z, bias)]
    y = selective_scan_momentum_fn(*full[:6], z=full[6], delta_bias=full[7], **kw)
    y.backward(dout)
    a, b = sum(seg_lens[:rank]), sum(seg_lens[: rank + 1])
    seg = lambda t: t[:, a:b].contiguous()
    mine = [seg(x), seg(delta), A, seg(Bm), seg(Cm), Dk, seg(z), bias]
    mine = [t.clone().requires_grad_() for t in mine]
    ys = seq_sharded_selective_scan(*mine[:6], z=mine[6], delta_bias=mine[7], seg_lens=seg_lens,
                                    **kw)
    ys.backward(seg(dout))
    torch.cuda.synchronize()
    lo = 4e-3 if dtype == torch.bfloat16 else 1e-4
    errs = {"y": (rel(ys, seg(y)), lo)}
    for name, fg, mg in zip(["x", "delta", "A", "B", "C", "D", "z", "bias"], full, mine):
        want = fg.grad if name in ("A", "D", "bias") else seg(fg.grad)
        tol = 1e-4 if name in ("A", "D", "bias") else lo
        errs["d" + name] = (rel(mg.grad, want), tol)
    bad = {k: v for k, v in errs.items() if not v[0] <= v[1]}
    print(f"rank {rank} {dtype}: " + " ".join(f"{k}={v[0]:.1e}" for k, v in errs.items()), flush=True)
    return not bad


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = True
    try:
        for dtype in (torch.float32, torch.bfloat16):
            ok = run(dtype, rank, world, dev) and ok
        flag = torch.tensor([0 if ok else 1], device=dev)
        dist.all_reduce(flag)
        ok = int(flag.item()) == 0
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
