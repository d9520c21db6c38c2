#!/usr/bin/env python
"""Benchmark of the momentum selective scan hot path on B200.

Workload (one "step"): the scan of a 4-layer MambaMomentum stack, forward and
backward -- per layer B=32 sequences, L=1024, D=256 channels (d_model 128 x
expand 2), N=16 states, with the block's softplus(delta + bias) and SiLU(z) gate
fused into the kernels.  Metric: scan elements (B*L*D*N) per second, fwd+bwd,
summed over all GPUs.  Multi-GPU runs are batch-sharded (weak scaling): every
rank scans its own 32 sequences per layer; the data path has no collective.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Rank 0 prints ONE JSON line.  ``--impl reference`` times the CPU restatement
of the reference algorithm (oracle/, fp32 variant, all host threads) on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "scan elements/s (B·L·D·N) fwd+bwd and HBM GB/s vs peak at 1/2/4/8 B200"
UNIT = "elements/s"

# workload shape
BSZ, SEQ, DIM, DST, LAYERS = 32, 1024, 256, 16, 4
BETA, ALPHA = 0.6, 1.0
ELEMS_PER_LAYER = BSZ * SEQ * DIM * DST

CONFIG = {
    "workload": "MambaMomentum 4-layer stack scan fwd+bwd (d_model 128, expand 2, d_state 16): "
                "B=32 L=1024 D=256 N=16 per layer, softplus(delta+bias) and SiLU(z) gate fused",
    "batch": BSZ, "seqlen": SEQ, "dim": DIM, "dstate": DST, "layers": LAYERS,
    "beta": BETA, "alpha": ALPHA,
    "l2": "inputs larger than L2: 4 layers x 138 MB of scan inputs per step",
}


def fwd_bytes(Bsz=BSZ, L=SEQ, D=DIM, N=DST):
    """Algorithmic bytes of one forward launch: read x, delta, z, B, C, A, D, bias;
    write out."""
    return 4 * (4 * Bsz * L * D + 2 * Bsz * L * N + D * N + 2 * D)


def bwd_bytes(Bsz=BSZ, L=SEQ, D=DIM, N=DST):
    """Algorithmic bytes of one backward launch: read x, delta, z, dout, B, C, A, D,
    bias; write dx, ddelta, dz, dB, dC, dA, dD, dbias."""
    return 4 * (7 * Bsz * L * D + 4 * Bsz * L * N + 2 * D * N + 4 * D)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(name="mmscan_bwd_traffic.json"):
    """DRAM bytes per backward launch (or call) from the committed ncu capture, if any."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return None


def max_over_ranks(ms: float, world: int, device=None) -> float:
    """Largest per-rank duration (the job's time); identity on one rank."""
    if world <= 1:
        return float(ms)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(ms)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(elems_per_rank: float, world: int, ms_job: float) -> float:
    """Whole-job throughput: the units every rank processed over the slowest rank's time."""
    return elems_per_rank * world / (ms_job / 1e3)


# ---------------------------------------------------------------------------
# clocks sampler
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
class Layer:
    """Device-resident inputs, outputs and checkpoint workspace of one layer."""

    def __init__(self, torch, lib, dev, gen, Bsz=BSZ):
        f = torch.float32
        self.Bsz = Bsz
        self.x = torch.randn(Bsz, SEQ, DIM, device=dev, generator=gen)
        self.delta = 0.5 * torch.randn(Bsz, SEQ, DIM, device=dev, generator=gen)  # raw dt_proj out
        self.z = torch.randn(Bsz, SEQ, DIM, device=dev, generator=gen)
        self.B = torch.randn(Bsz, SEQ, DST, device=dev, generator=gen)
        self.C = torch.randn(Bsz, SEQ, DST, device=dev, generator=gen)
        self.A = -torch.arange(1, DST + 1, device=dev, dtype=f).repeat(DIM, 1)
        self.D = torch.ones(DIM, device=dev)
        dt = torch.exp(torch.rand(DIM, device=dev, generator=gen) * (math.log(0.1) - math.log(1e-3))
                       + math.log(1e-3))
        self.bias = dt + torch.log(-torch.expm1(-dt))          # inverse softplus, as the block
        self.dout = torch.randn(Bsz, SEQ, DIM, device=dev, generator=gen)
        self.out = torch.empty(Bsz, SEQ, DIM, device=dev)
        self.ckpt = torch.empty(lib.mmb_mmscan_ckpt_floats(Bsz, SEQ, DIM, DST), device=dev)
        self.dx = torch.empty_like(self.x)
        self.ddelta = torch.empty_like(self.x)
        self.dz = torch.empty_like(self.x)
        self.dB = torch.empty_like(self.B)
        self.dC = torch.empty_like(self.C)
        self.dA = torch.empty_like(self.A)
        self.dD = torch.empty_like(self.D)
        self.dbias = torch.empty_like(self.D)


def make_desc(_lib, Bsz):
    d = _lib.MMScanDesc()
    d.batch, d.seqlen, d.dim, d.dstate = Bsz, SEQ, DIM, DST
    d.x_stride[:] = (SEQ * DIM, DIM)
    d.delta_stride[:] = (SEQ * DIM, DIM)
    d.z_stride[:] = (SEQ * DIM, DIM)
    d.B_stride[:] = (SEQ * DST, DST)
    d.C_stride[:] = (SEQ * DST, DST)
    d.beta, d.alpha, d.delta_softplus = BETA, ALPHA, 1
    return d


def run_b200(args):
    import torch
    import torch.distributed as dist

    from momentummamba_b200 import _lib
    from momentummamba_b200.selective_scan import selective_scan_momentum_fn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    lib = _lib.load()
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    bsz = args.batch if args.kernels_only else BSZ
    layers = [Layer(torch, lib, dev, gen, Bsz=bsz) for _ in range(LAYERS)]
    desc = make_desc(_lib, bsz)
    P = _lib.ptr

    def fwd(ly, stream):
        st = lib.mmb_mmscan_fwd(desc, P(ly.x), P(ly.delta), P(ly.A), P(ly.B), P(ly.C), P(ly.D),
                                P(ly.z), P(ly.bias), P(ly.out), P(ly.ckpt), stream)
        _lib.check(st, "fwd")

    def bwd(ly, stream):
        st = lib.mmb_mmscan_bwd(desc, P(ly.x), P(ly.delta), P(ly.A), P(ly.B), P(ly.C), P(ly.D),
                                P(ly.z), P(ly.bias), P(ly.ckpt), P(ly.dout), P(ly.dx),
                                P(ly.ddelta), P(ly.dA), P(ly.dB), P(ly.dC), P(ly.dD), P(ly.dz),
                                P(ly.dbias), stream)
        _lib.check(st, "bwd")

    def step():
        s = _lib.stream_of(layers[0].x)
        for ly in layers:
            fwd(ly, s)
            bwd(ly, s)

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (also sets the kernels' shared-memory attributes before capture)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if args.kernels_only:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.destroy_process_group()
        return None

    launch = "eager"
    graph = None
    if not args.no_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(graph, stream=s):
                    step()
            torch.cuda.current_stream().wait_stream(s)
            graph.replay()
            torch.cuda.synchronize()
            launch = "cuda graph"
        except Exception as e:  # capture unsupported: stay eager, say so
            graph = None
            launch = f"eager (graph capture failed: {type(e).__name__})"

    run = graph.replay if graph is not None else step
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()

    sampler = ClockSampler(local) if (rank == 0 and not args.no_clocks) else None
    if sampler:  # before the barrier, so that every rank starts the timed steps together
        sampler.start()
        time.sleep(0.5)
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    value = job_rate(ELEMS_PER_LAYER * LAYERS * args.steps, world, ms)

    # per-kernel durations (CUDA events on the launching stream), for the roofline
    ly = layers[0]
    s = _lib.stream_of(ly.x)
    cs = torch.cuda.current_stream()
    reps = 20
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(2 * reps)]
    for i in range(reps):
        lyr = layers[i % LAYERS]
        evs[2 * i][0].record(cs)
        fwd(lyr, s)
        evs[2 * i][1].record(cs)
        evs[2 * i + 1][0].record(cs)
        bwd(lyr, s)
        evs[2 * i + 1][1].record(cs)
    torch.cuda.synchronize()
    t_fwd = statistics.mean(evs[2 * i][0].elapsed_time(evs[2 * i][1]) for i in range(reps))
    t_bwd = statistics.mean(evs[2 * i + 1][0].elapsed_time(evs[2 * i + 1][1]) for i in range(reps))

    # end to end through the public autograd API with host buffers
    if world > 1:
        dist.barrier()
    e2e = run_e2e(torch, selective_scan_momentum_fn, dev, layers, args)
    e2e_ms = max_over_ranks(e2e["ms_per_step"], world, dev)
    e2e["ms_per_step"] = e2e_ms
    e2e["value"] = job_rate(ELEMS_PER_LAYER * LAYERS, world, e2e_ms)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(budget_s=args.cpu_budget)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None

    peak, peak_kind = load_peaks()
    bwd_b = bwd_bytes()
    fwd_b = fwd_bytes()
    achieved = bwd_b / (t_bwd / 1e3) / 1e9
    traffic = load_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(CONFIG, parallelism=f"batch-sharded x{world} (no data-path collective)",
                       launch=launch),
        "roofline": {
            "kernel": "mmscan_bwd_kernel<16>", "bound": "hbm", "achieved": achieved,
            "peak": peak, "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
            "algorithmic_bytes": bwd_b, "ms_per_launch": t_bwd,
        },
        "kernels": {
            "mmscan_fwd_kernel<16>": {"ms": t_fwd, "algorithmic_bytes": fwd_b,
                                      "GB/s": fwd_b / (t_fwd / 1e3) / 1e9,
                                      "frac": fwd_b / (t_fwd / 1e3) / 1e9 / peak},
            "mmscan_bwd_kernel<16>": {"ms": t_bwd, "algorithmic_bytes": bwd_b,
                                      "GB/s": achieved, "frac": achieved / peak},
        },
        "hbm_gbs_step": LAYERS * (fwd_b + bwd_b) * args.steps / (ms / 1e3) / 1e9,
        "e2e": e2e,
        "gpu_launches": 3 * LAYERS * args.steps,  # per layer: forward, clearing of the sums, backward
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    return line


def run_e2e(torch, fn, dev, layers, args, steps=8):
    """Same metric through selective_scan_momentum_fn + autograd, with each
    layer's inputs copied in from pinned host memory and all its outputs copied
    back every step.  The copies run on two side streams so that the next
    layer's inputs come in while the previous layer's outputs go out (PCIe is
    full duplex), and a step's uploads may start while the previous step's
    outputs still go out (steady state of a stream of batches); the scans run on
    the current stream in layer order.  The timed region ends after the last
    step's outputs reached the host."""
    host_in, host_out = [], []
    for ly in layers:
        host_in.append({k: getattr(ly, k).cpu().pin_memory()
                        for k in ("x", "delta", "z", "B", "C", "dout")})
        host_out.append({k: torch.empty(getattr(ly, k).shape, pin_memory=True)
                         for k in ("out", "dx", "ddelta", "dz", "dB", "dC", "dA", "dD", "dbias")})
    A, D, bias = layers[0].A, layers[0].D, layers[0].bias
    h2d = sum(t.numel() * 4 for t in host_in[0].values()) * LAYERS
    d2h = sum(t.numel() * 4 for t in host_out[0].values()) * LAYERS
    comp = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)

    def one():
        dev_in = [None] * LAYERS

        def fetch(i):
            with torch.cuda.stream(s_in):
                dev_in[i] = {k: v.to(dev, non_blocking=True) for k, v in host_in[i].items()}
                ev = torch.cuda.Event()
                ev.record(s_in)
            return ev

        ready = fetch(0)
        for i in range(LAYERS):
            comp.wait_event(ready)
            d = dev_in[i]
            for t in d.values():
                t.record_stream(comp)
            if i + 1 < LAYERS:
                ready = fetch(i + 1)
            ins = [d["x"].requires_grad_(True), d["delta"].requires_grad_(True),
                   A.detach().requires_grad_(True), d["B"].requires_grad_(True),
                   d["C"].requires_grad_(True), D.detach().requires_grad_(True),
                   d["z"].requires_grad_(True), bias.detach().requires_grad_(True)]
            y = fn(ins[0], ins[1], ins[2], ins[3], ins[4], ins[5], z=ins[6], delta_bias=ins[7],
                   delta_softplus=True, beta=BETA, alpha=ALPHA)
            gx, gd, gA, gB, gC, gD, gz, gb = torch.autograd.grad(y, ins, d["dout"])
            done = torch.cuda.Event()
            done.record(comp)
            outs = (("out", y), ("dx", gx), ("ddelta", gd), ("dz", gz), ("dB", gB), ("dC", gC),
                    ("dA", gA), ("dD", gD), ("dbias", gb))
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                for k, v in outs:
                    v = v.detach()
                    v.record_stream(s_out)
                    host_out[i][k].copy_(v, non_blocking=True)

    one()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    s_in.wait_stream(comp)
    s_out.wait_stream(comp)
    for _ in range(steps):
        one()
    comp.wait_stream(s_out)
    e1.record(comp)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"value": ELEMS_PER_LAYER * LAYERS / (ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms,
            "steps": steps, "api": "selective_scan_momentum_fn + torch.autograd.grad",
            "copies": "pinned host buffers; inputs of layer i+1 (and of the next step) in "
                      "while outputs of layer i go out (two copy streams)"}


# ---------------------------------------------------------------------------
# CPU (oracle restatement of the reference algorithm)
# ---------------------------------------------------------------------------
def cpu_inputs(np, nseq, seed=0):
    rng = np.random.default_rng(seed)
    f = np.float32
    x = rng.standard_normal((nseq, SEQ, DIM), dtype=f)
    delta = (0.5 * rng.standard_normal((nseq, SEQ, DIM))).astype(f)
    z = rng.standard_normal((nseq, SEQ, DIM), dtype=f)
    B = rng.standard_normal((nseq, SEQ, DST), dtype=f)
    C = rng.standard_normal((nseq, SEQ, DST), dtype=f)
    A = -np.tile(np.arange(1, DST + 1, dtype=f), (DIM, 1))
    D = np.ones(DIM, f)
    dt = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), DIM))
    bias = (dt + np.log(-np.expm1(-dt))).astype(f)
    dout = rng.standard_normal((nseq, SEQ, DIM), dtype=f)
    return x, delta, A, B, C, D, z, bias, dout


def cpu_scan_layer(oracle, inp):
    x, delta, A, B, C, D, z, bias, dout = inp
    oracle.mmscan_fwd(x, delta, A, B, C, D, z, bias, True, BETA, ALPHA, prec="f32")
    oracle.mmscan_bwd(x, delta, A, B, C, D, z, bias, True, BETA, ALPHA, dout, prec="f32")


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(budget_s=15.0):
    """Time the fp32 oracle (the reference recurrence restated in C) on the host
    cores: whole layers of 4 sequences each, repeated until ~budget_s."""
    import numpy as np

    import oracle
    cores = cpu_threads()
    oracle.set_num_threads(cores)
    nseq = 4
    inp = cpu_inputs(np, nseq)
    cpu_scan_layer(oracle, inp)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        cpu_scan_layer(oracle, inp)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    elems = n * nseq * SEQ * DIM * DST
    return {"value": elems / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} layer passes (fwd+bwd) of {nseq} of the {BSZ} sequences, "
                      f"{dt:.1f} s of CPU time; fp32 oracle/scan_oracle.c, OpenMP"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    import numpy as np

    import oracle
    cores = cpu_threads()
    oracle.set_num_threads(cores)
    # size each step so that warm-up + steps take about a minute
    probe = cpu_inputs(np, 1)
    t0 = time.perf_counter()
    cpu_scan_layer(oracle, probe)
    t_seq = time.perf_counter() - t0
    total = max(1, args.steps + args.warmup)
    nseq = int(max(1, min(BSZ, round(60.0 / (total * max(t_seq, 1e-3))))))
    inp = cpu_inputs(np, nseq)
    for _ in range(args.warmup):
        cpu_scan_layer(oracle, inp)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_scan_layer(oracle, inp)
    dt = time.perf_counter() - t0
    elems = args.steps * nseq * SEQ * DIM * DST
    value = elems / dt
    sample = (f"each step: one layer's scan fwd+bwd on {nseq} of the {BSZ} sequences "
              f"({nseq * SEQ * DIM * DST} elements); fp32 oracle/scan_oracle.c, OpenMP")
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": dict(CONFIG, parallelism="host cores (rank 0 only)"),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# long-sequence workload: one sequence split along time across the ranks
# ---------------------------------------------------------------------------
LONG = dict(batch=8, seqlen=65536, dim=2048, dstate=16, beta=0.9, alpha=1.0)


def long_bytes(Bsz, L, D, N):
    """Algorithmic bytes of one fwd+bwd over (Bsz, L) with bf16 activations:
    fwd reads x, delta, B, C and writes y; bwd reads x, delta, B, C, dy and
    writes dx, ddelta, dB, dC (fp32 sums counted at 4 bytes)."""
    fwd = 2 * (3 * Bsz * L * D + 2 * Bsz * L * N) + 4 * (D * N + D)
    bwd = 2 * (5 * Bsz * L * D + 2 * Bsz * L * N) + 4 * (2 * Bsz * L * N + 2 * D * N + 2 * D)
    return fwd, bwd


def run_long(args):
    """B=8, L=65536, D=2048, N=16 with bf16 activations, fp32 state: the
    sequence is split into WORLD_SIZE contiguous segments, one per rank
    (segment summaries all-gathered over NCCL, carries folded locally).  Total
    work is fixed (strong scaling)."""
    import datetime

    import torch
    import torch.distributed as dist

    from momentummamba_b200.selective_scan import ScanCall
    from momentummamba_b200.seqshard import SegmentOps as ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    Bsz, L, D, N = (LONG[k] for k in ("batch", "seqlen", "dim", "dstate"))
    beta, alpha = LONG["beta"], LONG["alpha"]
    Lr = L // world
    seg_lens = [Lr] * world
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    bf = torch.bfloat16
    x = torch.randn(Bsz, Lr, D, device=dev, generator=gen).to(bf)
    delta = torch.nn.functional.softplus(
        0.5 * torch.randn(Bsz, Lr, D, device=dev, generator=gen) - 2.0).to(bf)
    Bm = torch.randn(Bsz, Lr, N, device=dev, generator=gen).to(bf)
    Cm = torch.randn(Bsz, Lr, N, device=dev, generator=gen).to(bf)
    A = -torch.arange(1, N + 1, device=dev, dtype=torch.float32).repeat(D, 1)
    Dk = torch.ones(D, device=dev)
    dout = torch.randn(Bsz, Lr, D, device=dev, generator=gen).to(bf)
    call = ScanCall(x, delta, A, Bm, Cm, Dk, None, None, False, beta, alpha)
    assert call.adtype == bf

    def gather(t):
        out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), device=dev)
        dist.all_gather_into_tensor(out, t)
        return out.view((world,) + tuple(t.shape))

    marks = {}

    def mark(name):
        if args.phases:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            marks.setdefault(name, []).append(e)

    def step():
        mark("start")
        if world > 1:
            summ = gather(ops.fwd_summary(call))
            state = ops.carry_fwd(summ, rank, seg_lens, beta) if rank > 0 else None
        else:
            summ, state = None, None
        mark("fwd_carry")
        _, ckpt = ops.forward(call, state, True)
        mark("fwd")
        gstate = None
        if world > 1:
            gs = ops.bwd_summary(call, dout)
            gsumm = gather(gs)
            gstate = ops.carry_bwd(summ, gsumm, rank, seg_lens, beta) if rank < world - 1 else None
        mark("bwd_carry")
        g = ops.backward(call, ckpt, dout, gstate)
        if world > 1:
            flat = torch.cat([g[2].reshape(-1), g[5]])
            dist.all_reduce(flat)
        mark("bwd")

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    marks.clear()
    sampler = ClockSampler(local) if (rank == 0 and not args.no_clocks) else None
    if sampler:  # before the barrier, so that every rank starts the timed steps together
        sampler.start()
        time.sleep(0.5)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    phases = None
    if args.phases and marks:
        names = ["start", "fwd_carry", "fwd", "bwd_carry", "bwd"]
        phases = {}
        for a, b in zip(names[:-1], names[1:]):
            t = statistics.mean(marks[a][i].elapsed_time(marks[b][i]) for i in range(args.steps))
            phases[b] = max_over_ranks(t, world, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    elems = Bsz * L * D * N
    fb, bb = long_bytes(Bsz, Lr, D, N)
    peak, peak_kind = load_peaks()
    ms_step = ms / args.steps
    achieved = (fb + bb) / (ms_step / 1e3) / 1e9  # per GPU: its segment's bytes over the step
    return {
        "metric": METRIC, "value": elems / (ms_step / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "long-sequence scan fwd+bwd: B=8 L=65536 D=2048 N=16, bf16 "
                               "activations, fp32 state; x ~ N(0,1), delta = softplus(0.5 N(0,1) - 2), "
                               "A[d,n] = -(n+1), D = 1, beta 0.9, alpha 1",
                   "parallelism": f"sequence-sharded x{world} (segment summaries all-gathered)",
                   "segment": Lr, "l2": "inputs larger than L2 (2.1 GB per bf16 activation)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s", "frac": achieved / peak,
                     "algorithmic_bytes_per_gpu_step": fb + bb, "traffic": None,
                     "scope": "whole step per GPU (fwd+bwd kernels, carries, collectives)"},
        "phases_ms": phases,
        # rank 0: forward, clearing of the backward's sums, backward; with segments also
        # both summaries and the adjoint fold
        "gpu_launches": (3 if world == 1 else 6) * args.steps,
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------
# LinOSS layer scan workload (IM and IMEX discretisations)
# ---------------------------------------------------------------------------
LINOSS = dict(batch=16, seqlen=4096, osc=256)


def run_linoss(args):
    """The LinOSS layer scan (LinOSS_pytorch.py:153-239, time-invariant 2x2
    transition built in-kernel) forward + backward for IM and IMEX at B=16
    L=4096 P=256 with complex Bu ~ N(0,1), A ~ U[0,1], step = exp(U[ln 1e-3,
    ln 1e-1]).  One step = IM fwd + bwd and IMEX fwd + bwd; elements = B L P
    oscillator steps per discretisation.  Batch-sharded over ranks (weak)."""
    import datetime

    import torch
    import torch.distributed as dist

    from momentummamba_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    Bsz, L, P = LINOSS["batch"], LINOSS["seqlen"], LINOSS["osc"]
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    A = torch.rand(P, device=dev, generator=g)
    step = torch.exp(torch.rand(P, device=dev, generator=g) * (math.log(0.1) - math.log(1e-3))
                     + math.log(1e-3))
    Bu = torch.randn(Bsz, L, P, 2, device=dev, generator=g)
    dx2 = torch.randn(Bsz, L, P, 2, device=dev, generator=g)
    x2 = torch.empty_like(Bu)
    dBu = torch.empty_like(Bu)
    dA = torch.empty_like(A)
    ds = torch.empty_like(step)
    works = [torch.empty(lib.mmb_linoss_work_floats(Bsz, L, P), device=dev) for _ in range(2)]
    Pp = _lib.ptr

    def fwd(disc):  # on the current stream (the capture stream while capturing)
        _lib.check(lib.mmb_linoss_fwd(disc, Bsz, L, P, Pp(A), Pp(step), Pp(Bu), Pp(x2),
                                      Pp(works[disc]), _lib.stream_of(Bu)), "linoss fwd")

    def bwd(disc):
        _lib.check(lib.mmb_linoss_bwd(disc, Bsz, L, P, Pp(A), Pp(step), Pp(Bu), Pp(dx2), Pp(dBu),
                                      Pp(dA), Pp(ds), Pp(works[disc]), _lib.stream_of(Bu)),
                   "linoss bwd")

    def stepfn():
        for disc in (0, 1):   # IM, IMEX
            fwd(disc)
            bwd(disc)

    for _ in range(max(3, args.warmup)):
        stepfn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device=dev)
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            stepfn()
    torch.cuda.current_stream().wait_stream(cs)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if (rank == 0 and not args.no_clocks) else None
    if sampler:
        sampler.start()
        time.sleep(0.5)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    # per-kernel durations
    reps = 10
    t = {}
    cur = torch.cuda.current_stream()
    for name, fn in (("fwd_IM", lambda: fwd(0)), ("bwd_IM", lambda: bwd(0)),
                     ("fwd_IMEX", lambda: fwd(1)), ("bwd_IMEX", lambda: bwd(1))):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for a, b in evs:
            a.record(cur)
            fn()
            b.record(cur)
        torch.cuda.synchronize()
        t[name] = statistics.mean(a.elapsed_time(b) for a, b in evs)
    del graph
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    elems = Bsz * L * P
    fwd_b = elems * 16 + 2 * P * 4          # read Bu, write x2 (complex fp32)
    bwd_b = elems * 24 + 4 * P * 4          # read Bu, dx2; write dBu
    peak, peak_kind = load_peaks()
    achieved = bwd_b / (t["bwd_IM"] / 1e3) / 1e9
    tr = load_traffic("linoss_bwd_traffic.json")
    return {
        "metric": METRIC, "value": job_rate(2 * elems * args.steps, world, ms), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "LinOSS layer scan fwd+bwd, IM and IMEX: B=16 L=4096 P=256, "
                               "complex Bu ~ N(0,1), A ~ U[0,1], step = exp(U[ln 1e-3, ln 1e-1]); "
                               "elements = B*L*P oscillator steps per discretisation",
                   "parallelism": f"batch-sharded x{world}", "launch": "cuda graph",
                   "l2": "inputs larger than L2 (Bu, dx2 134 MB each; 1.3 GB of algorithmic traffic per step)"},
        "roofline": {"kernel": "lin_bwd (IM): summary + carry + final + params launches",
                     "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s", "frac": achieved / peak,
                     "algorithmic_bytes": bwd_b, "ms_per_launch": t["bwd_IM"],
                     "traffic": tr["dram_bytes_per_call"] if tr else None},
        "kernels": {k: {"ms": v, "algorithmic_bytes": fwd_b if k.startswith("fwd") else bwd_b,
                        "GB/s": (fwd_b if k.startswith("fwd") else bwd_b) / (v / 1e3) / 1e9}
                    for k, v in t.items()},
        # per discretisation: forward summary, carry, final; backward summary, carry,
        # final, parameter chain rule
        "gpu_launches": 14 * args.steps,
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------
# row-form and PScan-layout scans (the reference's materialised-tensor paths)
# ---------------------------------------------------------------------------
def run_rows(args):
    """The momentum row scan (momentum_scan_cuda.py:204-253: R = B*D*N rows of L
    steps) and the diagonal scan in the PScan layout (pscan.py:43-234: (B, L,
    D*N)) forward + backward at the stack's size (B=32, L=1024, D=256, N=16:
    134,217,728 elements each).  One step = rows fwd + bwd, then pscan fwd + bwd;
    elements = the rows scan's (the line's value), per-kernel GB/s for both.
    Batch-sharded replicas over ranks (weak)."""
    import datetime

    import torch
    import torch.distributed as dist

    from momentummamba_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    R, L, M = BSZ * DIM * DST, SEQ, DIM * DST
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    a = torch.exp(-torch.rand(R, L, device=dev, generator=g) * 0.2)     # decay factors in (0.82, 1]
    u = torch.randn(R, L, device=dev, generator=g)
    gr = torch.randn(R, L, device=dev, generator=g)
    h, da, du = torch.empty_like(a), torch.empty_like(a), torch.empty_like(a)
    A3, X3, G3 = a.view(BSZ, L, M), u.view(BSZ, L, M), gr.view(BSZ, L, M)  # same bytes, PScan layout
    H3, dA3, dX3 = torch.empty_like(A3), torch.empty_like(A3), torch.empty_like(A3)
    Pp = _lib.ptr

    def rows_fwd():
        _lib.check(lib.mmb_rows_fwd(R, L, Pp(a), BETA, Pp(u), Pp(h), None, _lib.stream_of(a)),
                   "rows fwd")

    def rows_bwd():
        _lib.check(lib.mmb_rows_bwd(R, L, Pp(gr), Pp(a), BETA, Pp(h), Pp(da), Pp(du),
                                    _lib.stream_of(a)), "rows bwd")

    def ps_fwd():
        _lib.check(lib.mmb_pscan_fwd(BSZ, L, M, Pp(A3), Pp(X3), Pp(H3), _lib.stream_of(a)),
                   "pscan fwd")

    def ps_bwd():
        _lib.check(lib.mmb_pscan_bwd(BSZ, L, M, Pp(A3), Pp(H3), Pp(G3), Pp(dA3), Pp(dX3),
                                     _lib.stream_of(a)), "pscan bwd")

    def stepfn():
        rows_fwd()
        rows_bwd()
        ps_fwd()
        ps_bwd()

    for _ in range(max(3, args.warmup)):
        stepfn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device=dev)
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            stepfn()
    torch.cuda.current_stream().wait_stream(cs)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if (rank == 0 and not args.no_clocks) else None
    if sampler:
        sampler.start()
        time.sleep(0.5)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    reps = 10
    t = {}
    cur = torch.cuda.current_stream()
    for name, fn in (("rows_fwd", rows_fwd), ("rows_bwd", rows_bwd), ("pscan_fwd", ps_fwd),
                     ("pscan_bwd", ps_bwd)):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for e_a, e_b in evs:
            e_a.record(cur)
            fn()
            e_b.record(cur)
        torch.cuda.synchronize()
        t[name] = statistics.mean(x.elapsed_time(y) for x, y in evs)
    del graph
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    elems = R * L
    nbytes = {"rows_fwd": 12 * elems, "rows_bwd": 20 * elems,   # a, u -> h; g, a, h -> da, du
              "pscan_fwd": 12 * elems, "pscan_bwd": 20 * elems}  # A, X -> H; A, H, G -> dA, dX
    peak, peak_kind = load_peaks()
    kern = {k: {"ms": v, "algorithmic_bytes": nbytes[k], "GB/s": nbytes[k] / (v / 1e3) / 1e9,
                "frac": nbytes[k] / (v / 1e3) / 1e9 / peak} for k, v in t.items()}
    return {
        "metric": METRIC, "value": job_rate(elems * args.steps, world, ms), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "materialised-tensor scans at the stack's size: momentum row scan "
                               "(R=131072 rows x L=1024, beta 0.6) and PScan-layout diagonal scan "
                               "(B=32 L=1024 M=4096), fwd+bwd each; value = row-scan elements/s "
                               "over the whole step",
                   "parallelism": f"batch-sharded x{world}", "launch": "cuda graph",
                   "l2": "inputs larger than L2 (537 MB per tensor)"},
        "roofline": {"kernel": "rows_bwd", "bound": "hbm", "achieved": kern["rows_bwd"]["GB/s"],
                     "peak": peak, "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s",
                     "frac": kern["rows_bwd"]["frac"], "algorithmic_bytes": nbytes["rows_bwd"],
                     "ms_per_launch": t["rows_bwd"], "traffic": None},
        "kernels": kern,
        "gpu_launches": 4 * args.steps,
        "clocks": clocks,
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--kernels-only", action="store_true",
                    help="run warm-up and steps eagerly and exit (for profiler captures)")
    ap.add_argument("--batch", type=int, default=BSZ,
                    help="sequences per layer (profiling only; the benchmark line uses 32)")
    ap.add_argument("--workload", choices=["stack", "long", "linoss", "rows"], default="stack",
                    help="stack: the 4-layer MambaMomentum scan (batch-sharded, the benchmark "
                         "line); long: B=8 L=65536 D=2048 bf16, sequence-sharded; linoss: the "
                         "LinOSS layer scan, IM and IMEX, B=16 L=4096 P=256; rows: the "
                         "row-form and PScan-layout scans at the stack's size")
    ap.add_argument("--phases", action="store_true",
                    help="long workload: also time each phase (adds events to the step)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        line = run_reference(args)
    elif args.workload == "long":
        line = run_long(args)
    elif args.workload == "linoss":
        line = run_linoss(args)
    elif args.workload == "rows":
        line = run_rows(args)
    else:
        line = run_b200(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
