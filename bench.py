#!/usr/bin/env python
"""Benchmark of the momentum selective scan hot path on B200.

Default line (one "step"): the scan of the momentum-Mamba sequence classifier,
forward and backward -- 6 MambaMomentum layers, each B=256 sequences, T=300,
D=512 channels (d_model 256 x expand 2), N=16 states, with the block's
softplus(delta + bias) and SiLU(z) gate fused into the kernels, fp32.  Metric:
scan elements (B*T*D*N) per second, fwd+bwd, whole job.  ``--gpus N`` splits
the 256 sequences over the ranks (B = 256/N each, strong scaling): sequences
are independent, so the data path has no collective.

Extra keys of the same line (each with its own roofline):
  * ``stack_cfg1``: the 4-layer stack of d_model 128 (B=32 L=1024 D=256 N=16);
  * ``time_chunks``: 4 layers of B=2 L=8192 D=256 N=16, too few channels to
                    fill the GPU, so each call splits the sequence into time
                    chunks scanned by separate CTAs (with the unsplit calls'
                    times beside);
  * ``long_seq``:   B=8 L=65536 D=2048 N=16 in bf16, split along time over the
                    ranks (segment summaries all-gathered over NCCL);
  * ``linoss``:     the LinOSS layer scan, IM and IMEX, B=16 L=4096 P=256;
  * ``linoss_layer``: the whole LinOSS layer (tensor-core contractions + scan)
                    at H=128, with the cuBLAS-contraction layer's time beside;
  * ``rows``:       the row-form and PScan-layout scans at the stack's size.
On N > 1 GPUs only ``long_seq`` runs beside the default line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload classifier|stack|chunks|long|linoss|linoss_layer|rows] [--no-extras]

Rank 0 prints ONE JSON line.  ``--impl reference`` times the CPU restatement
of the reference algorithm (oracle/, fp32 variant, all host threads) on a
bounded sample of the default workload.
"""
from __future__ import annotations

import argparse
import datetime
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
BETA, ALPHA = 0.6, 1.0

# momentum-Mamba sequence classifier: 6 layers of d_model 256, expand 2
CLASSIFIER = dict(batch=256, seqlen=300, dim=512, dstate=16, layers=6)
# MambaMomentum stack of d_model 128, expand 2: 4 layers
STACK1 = dict(batch=32, seqlen=1024, dim=256, dstate=16, layers=4)
# short batch of long sequences (d_model 128, expand 2): 512 channels give the
# GPU 64 warps, so each call splits along time (chunks scanned by separate CTAs)
CHUNKED = dict(batch=2, seqlen=8192, dim=256, dstate=16, layers=4, compare_unsplit=True)


def fwd_bytes(Bsz, L, D, N):
    """Algorithmic bytes of one forward launch: read x, delta, z, B, C, A, D, bias;
    write out."""
    return 4 * (4 * Bsz * L * D + 2 * Bsz * L * N + D * N + 2 * D)


def bwd_bytes(Bsz, L, D, N):
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


def load_traffic(name, key=None):
    """DRAM bytes per launch (or call) from a committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            d = json.load(f)
        return d[key] if key else d
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


def ctx_max(ms: float, ctx) -> float:
    return max_over_ranks(ms, ctx.world, ctx.dev)


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


class Ctx:
    """Process-wide state of one benchmark run (one process per GPU)."""

    def __init__(self, args):
        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = None

    def init_gpu(self):
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def close(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def timed_region(ctx, run, steps):
    """Barrier + synchronize on both sides, CUDA events around `steps` calls of
    run() on the current stream, clocks sampled meanwhile on rank 0.  Returns
    (max-over-ranks ms, clocks)."""
    import torch
    sampler = ClockSampler(ctx.local) if (ctx.rank == 0 and not ctx.args.no_clocks) else None
    if sampler:  # before the barrier, so that every rank starts the timed steps together
        sampler.start()
        time.sleep(0.5)
    ctx.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ctx.barrier()
    clocks = sampler.stop() if sampler else None
    return ctx_max(e0.elapsed_time(e1), ctx), clocks


def capture(ctx, fn):
    """One CUDA graph of fn() (the kernels' shared-memory attributes were set by
    eager warm-up calls before)."""
    import torch
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=ctx.dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    return graph


def launch_times(pairs, reps=10):
    """Mean CUDA-event duration of each named launch function, events recorded on
    the current stream (the stream the library launches on)."""
    import torch
    cur = torch.cuda.current_stream()
    out = {}
    for name, fn in pairs:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for a, b in evs:
            a.record(cur)
            fn()
            b.record(cur)
        torch.cuda.synchronize()
        out[name] = statistics.mean(a.elapsed_time(b) for a, b in evs)
    return out


# ---------------------------------------------------------------------------
# momentum scan stacks (the default classifier line and the d_model-128 stack)
# ---------------------------------------------------------------------------
class Layer:
    """Device-resident inputs, outputs and checkpoint workspace of one layer."""

    def __init__(self, torch, lib, dev, gen, Bsz, L, D, N):
        f = torch.float32
        self.shape = (Bsz, L, D, N)
        self.x = torch.randn(Bsz, L, D, device=dev, generator=gen)
        self.delta = 0.5 * torch.randn(Bsz, L, D, device=dev, generator=gen)  # raw dt_proj out
        self.z = torch.randn(Bsz, L, D, device=dev, generator=gen)
        self.B = torch.randn(Bsz, L, N, device=dev, generator=gen)
        self.C = torch.randn(Bsz, L, N, device=dev, generator=gen)
        self.A = -torch.arange(1, N + 1, device=dev, dtype=f).repeat(D, 1)
        self.D = torch.ones(D, device=dev)
        dt = torch.exp(torch.rand(D, device=dev, generator=gen) * (math.log(0.1) - math.log(1e-3))
                       + math.log(1e-3))
        self.bias = dt + torch.log(-torch.expm1(-dt))          # inverse softplus, as the block
        self.dout = torch.randn(Bsz, L, D, device=dev, generator=gen)
        self.out = torch.empty(Bsz, L, D, device=dev)
        self.ckpt = torch.empty(lib.mmb_mmscan_ckpt_floats(Bsz, L, D, N), device=dev)
        self.dx = torch.empty_like(self.x)
        self.ddelta = torch.empty_like(self.x)
        self.dz = torch.empty_like(self.x)
        self.dB = torch.empty_like(self.B)
        self.dC = torch.empty_like(self.C)
        self.dA = torch.empty_like(self.A)
        self.dD = torch.empty_like(self.D)
        self.dbias = torch.empty_like(self.D)


def make_desc(_lib, Bsz, L, D, N, time_chunk=0):
    d = _lib.MMScanDesc()
    d.time_chunk = time_chunk
    d.batch, d.seqlen, d.dim, d.dstate = Bsz, L, D, N
    d.x_stride[:] = (L * D, D)
    d.delta_stride[:] = (L * D, D)
    d.z_stride[:] = (L * D, D)
    d.B_stride[:] = (L * N, N)
    d.C_stride[:] = (L * N, N)
    d.beta, d.alpha, d.delta_softplus = BETA, ALPHA, 1
    return d


def run_stack(ctx, cfg, strong, steps, with_e2e, with_cpu, name):
    """Time the scan fwd+bwd of a stack of layers.  strong: the cfg batch is the
    whole job's, split over the ranks; else every rank runs the whole batch."""
    import torch

    from momentummamba_b200 import _lib
    from momentummamba_b200.selective_scan import selective_scan_momentum_fn

    args = ctx.args
    Btot, L, D, N, NL = (cfg[k] for k in ("batch", "seqlen", "dim", "dstate", "layers"))
    if strong:
        if Btot % ctx.world:
            raise SystemExit(f"batch {Btot} does not split over {ctx.world} ranks")
        Bsz = Btot // ctx.world
    else:
        Bsz = Btot
    if args.batch:  # profiling of a smaller case of the same kernels
        Bsz = args.batch
    lib = _lib.load()
    gen = torch.Generator(device=ctx.dev).manual_seed(1234 + ctx.rank)
    layers = [Layer(torch, lib, ctx.dev, gen, Bsz, L, D, N) for _ in range(NL)]
    desc = make_desc(_lib, Bsz, L, D, N)
    P = _lib.ptr

    def fwd(ly, dsc=desc):
        st = lib.mmb_mmscan_fwd(dsc, P(ly.x), P(ly.delta), P(ly.A), P(ly.B), P(ly.C), P(ly.D),
                                P(ly.z), P(ly.bias), P(ly.out), P(ly.ckpt), _lib.stream_of(ly.x))
        _lib.check(st, "fwd")

    def bwd(ly, dsc=desc):
        st = lib.mmb_mmscan_bwd(dsc, P(ly.x), P(ly.delta), P(ly.A), P(ly.B), P(ly.C), P(ly.D),
                                P(ly.z), P(ly.bias), P(ly.ckpt), P(ly.dout), P(ly.dx),
                                P(ly.ddelta), P(ly.dA), P(ly.dB), P(ly.dC), P(ly.dD), P(ly.dz),
                                P(ly.dbias), _lib.stream_of(ly.x))
        _lib.check(st, "bwd")

    def step():
        for ly in layers:
            fwd(ly)
            bwd(ly)

    # warm-up (also sets the kernels' shared-memory attributes before capture)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if args.kernels_only:  # eager launches only, for profiler captures
        for _ in range(steps):
            step()
        torch.cuda.synchronize()
        return None
    launch = "cuda graph"
    try:
        graph = capture(ctx, step)
        run = graph.replay
    except Exception as e:  # capture unsupported: stay eager, say so
        graph = None
        run = step
        launch = f"eager (graph capture failed: {type(e).__name__})"
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    ms, clocks = timed_region(ctx, run, steps)
    elems_layer = Bsz * L * D * N
    value = job_rate(elems_layer * NL * steps, ctx.world, ms)

    # per-launch durations of the layer kernels (CUDA events on the launching stream)
    t = launch_times([("fwd", lambda: fwd(layers[0])), ("bwd", lambda: bwd(layers[1]))], reps=10)
    t_fwd = ctx_max(t["fwd"], ctx)
    t_bwd = ctx_max(t["bwd"], ctx)
    unsplit = None
    if cfg.get("compare_unsplit"):
        # the same calls with the split along time turned off
        d1 = make_desc(_lib, Bsz, L, D, N, time_chunk=-1)
        u = launch_times([("fwd", lambda: fwd(layers[0], d1)), ("bwd", lambda: bwd(layers[1], d1))],
                         reps=5)
        unsplit = {"fwd_ms": ctx_max(u["fwd"], ctx), "bwd_ms": ctx_max(u["bwd"], ctx)}
    nch = -(-L // chunk_len(lib, _lib, desc))
    del graph

    e2e = None
    if with_e2e:
        ctx.barrier()
        e2e = run_e2e(torch, selective_scan_momentum_fn, ctx, layers, cfg)
    cpu = None
    if with_cpu and ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, budget_s=args.cpu_budget)
    del layers
    torch.cuda.empty_cache()
    if ctx.rank != 0:
        return None

    peak, peak_kind = load_peaks()
    fb, bb = fwd_bytes(Bsz, L, D, N), bwd_bytes(Bsz, L, D, N)
    achieved = bb / (t_bwd / 1e3) / 1e9
    traffic = load_traffic("mmscan_bwd_traffic.json", name)
    kb = bwd_kernel_name(Bsz, D, N, nch)
    workload = (f"{NL}-layer momentum-Mamba scan fwd+bwd (expand 2, d_state {N}): "
                f"B={Btot} L={L} D={D} N={N} per layer, softplus(delta+bias) and SiLU(z) "
                f"gate fused, fp32")
    if nch > 1:
        workload += (f"; each call split along time into {nch} chunks (summary, carry and "
                     f"full passes)")
    par = (f"batch split over {ctx.world} rank(s): {Bsz} sequences each, no data-path "
           f"collective" if strong else f"batch-sharded replicas x{ctx.world}: {Bsz} "
           f"sequences per rank, no data-path collective")
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ctx.world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload, "batch": Btot, "batch_per_rank": Bsz, "seqlen": L,
                   "dim": D, "dstate": N, "layers": NL, "beta": BETA, "alpha": ALPHA,
                   "parallelism": par, "launch": launch,
                   "l2": f"inputs larger than L2: {NL} layers x "
                         f"{fwd_bytes(Bsz, L, D, N) / 1e6:.0f} MB of scan inputs per step"},
        "roofline": {
            "kernel": (kb if nch == 1 else
                       f"backward call: clearing + summary + carry + {kb} "
                       f"over {nch} time chunks"),
            "bound": "hbm", "achieved": achieved,
            "peak": peak, "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
            "traffic_note": traffic.get("note") if traffic else None,
            "algorithmic_bytes": bb, "ms_per_launch": t_bwd,
        },
        "kernels": {
            f"mmscan_fwd_kernel<{N}>": {"ms": t_fwd, "algorithmic_bytes": fb,
                                        "GB/s": fb / (t_fwd / 1e3) / 1e9,
                                        "frac": fb / (t_fwd / 1e3) / 1e9 / peak},
            kb: {"ms": t_bwd, "algorithmic_bytes": bb,
                                        "GB/s": achieved, "frac": achieved / peak},
        },
        "hbm_gbs_step": NL * (fb + bb) * steps / (ms / 1e3) / 1e9,
        "time_chunks": nch,
        "unsplit": unsplit,
        "e2e": e2e,
        # per layer: forward, clearing of the backward's sums, backward; split
        # calls add a summary and a carry launch to each side
        "gpu_launches": (3 + (4 if nch > 1 else 0)) * NL * steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }


def bwd_kernel_name(Bsz, D, N, nch):
    """The backward kernel the library picks for an fp32 call with 4 states per
    thread: the two-channel kernel (256 / N channels per one-warp CTA) when its
    grid gives every one of the 148 SMs at least 6 CTAs, else the one-channel
    kernel."""
    ctas = -(-D // (256 // N)) * Bsz * nch
    two = 8 <= N <= 32 and ctas >= 148 * 6
    return f"mmscan_bwd2_kernel<{N}>" if two else f"mmscan_bwd_kernel<{N}>"


def chunk_len(lib, _lib, desc):
    """Steps per time chunk the library uses for desc (the sequence length when
    it does not split), from the workspace it asks for."""
    import ctypes
    Bsz, L, D, N = desc.batch, desc.seqlen, desc.dim, desc.dstate
    extra = lib.mmb_mmscan_workspace_floats(ctypes.byref(desc)) - Bsz * (-(-L // 8)) * D * N * 2
    nch = extra // (Bsz * D * N * 6) if extra else 1
    return -(-L // nch)


def run_e2e(torch, fn, ctx, layers, cfg, steps=4):
    """Same metric through selective_scan_momentum_fn + autograd, with each
    layer's inputs copied in from pinned host memory and all its outputs copied
    back every step.  The copies run on two side streams so that the next
    layer's inputs come in while the previous layer's outputs go out (PCIe is
    full duplex), and a step's uploads may start while the previous step's
    outputs still go out (steady state of a stream of batches); the scans run on
    the current stream in layer order.  Every layer reads the same pinned host
    inputs and writes the same pinned host outputs (one set of host buffers).
    The timed region ends after the last step's outputs reached the host."""
    dev = ctx.dev
    NL = len(layers)
    ly0 = layers[0]
    host_in = {k: getattr(ly0, k).cpu().pin_memory()
               for k in ("x", "delta", "z", "B", "C", "dout")}
    host_out = {k: torch.empty(getattr(ly0, k).shape, pin_memory=True)
                for k in ("out", "dx", "ddelta", "dz", "dB", "dC", "dA", "dD", "dbias")}
    A, D, bias = ly0.A, ly0.D, ly0.bias
    h2d = sum(t.numel() * 4 for t in host_in.values()) * NL
    d2h = sum(t.numel() * 4 for t in host_out.values()) * NL
    comp = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)
    Bsz, L, Dm, N = ly0.shape

    def one():
        dev_in = [None] * NL

        def fetch(i):
            with torch.cuda.stream(s_in):
                dev_in[i] = {k: v.to(dev, non_blocking=True) for k, v in host_in.items()}
                ev = torch.cuda.Event()
                ev.record(s_in)
            return ev

        ready = fetch(0)
        for i in range(NL):
            comp.wait_event(ready)
            d = dev_in[i]
            for t in d.values():
                t.record_stream(comp)
            if i + 1 < NL:
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
                    host_out[k].copy_(v, non_blocking=True)

    one()
    torch.cuda.synchronize()
    ctx.barrier()
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
    ms = ctx_max(e0.elapsed_time(e1) / steps, ctx)
    elems = Bsz * L * Dm * N * NL
    return {"value": job_rate(elems, ctx.world, ms), "unit": UNIT,
            "h2d_bytes_per_step": h2d * ctx.world, "d2h_bytes_per_step": d2h * ctx.world,
            "h2d_bytes_per_rank_step": h2d, "d2h_bytes_per_rank_step": d2h,
            "ms_per_step": ms, "steps": steps,
            "api": "selective_scan_momentum_fn + torch.autograd.grad",
            "copies": "pinned host buffers; inputs of layer i+1 (and of the next step) in "
                      "while outputs of layer i go out (two copy streams)"}


# ---------------------------------------------------------------------------
# CPU (oracle restatement of the reference algorithm)
# ---------------------------------------------------------------------------
def cpu_inputs(np, cfg, nseq, seed=0):
    L, D, N = cfg["seqlen"], cfg["dim"], cfg["dstate"]
    rng = np.random.default_rng(seed)
    f = np.float32
    x = rng.standard_normal((nseq, L, D), dtype=f)
    delta = (0.5 * rng.standard_normal((nseq, L, D))).astype(f)
    z = rng.standard_normal((nseq, L, D), dtype=f)
    B = rng.standard_normal((nseq, L, N), dtype=f)
    C = rng.standard_normal((nseq, L, N), dtype=f)
    A = -np.tile(np.arange(1, N + 1, dtype=f), (D, 1))
    Dv = np.ones(D, f)
    dt = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), D))
    bias = (dt + np.log(-np.expm1(-dt))).astype(f)
    dout = rng.standard_normal((nseq, L, D), dtype=f)
    return x, delta, A, B, C, Dv, z, bias, dout


def cpu_scan_layer(oracle, inp):
    x, delta, A, B, C, D, z, bias, dout = inp
    oracle.mmscan_fwd(x, delta, A, B, C, D, z, bias, True, BETA, ALPHA, prec="f32")
    oracle.mmscan_bwd(x, delta, A, B, C, D, z, bias, True, BETA, ALPHA, dout, prec="f32")


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(cfg, budget_s=15.0, nseq=None):
    """Time the fp32 oracle (the reference recurrence restated in C) on the host
    cores: whole layers of a few sequences each, repeated until ~budget_s."""
    import numpy as np

    import oracle
    cores = cpu_threads()
    oracle.set_num_threads(cores)
    L, D, N = cfg["seqlen"], cfg["dim"], cfg["dstate"]
    nseq = nseq or max(1, min(cfg["batch"], int(round(2e7 / (L * D * N)))))
    inp = cpu_inputs(np, cfg, nseq)
    cpu_scan_layer(oracle, inp)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        cpu_scan_layer(oracle, inp)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    elems = n * nseq * L * D * N
    return {"value": elems / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} layer passes (fwd+bwd) of {nseq} of the {cfg['batch']} sequences "
                      f"(L={L} D={D} N={N}), {dt:.1f} s of CPU time; fp32 oracle/scan_oracle.c, "
                      f"OpenMP"}


def run_reference(args):
    """The reference arm: the CPU restatement of the reference recurrence on the
    host cores, on the default workload's shapes (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    import numpy as np

    import oracle
    cfg = CLASSIFIER
    L, D, N = cfg["seqlen"], cfg["dim"], cfg["dstate"]
    cores = cpu_threads()
    oracle.set_num_threads(cores)
    # size each step so that warm-up + steps take about a minute
    probe = cpu_inputs(np, cfg, 4)
    t0 = time.perf_counter()
    cpu_scan_layer(oracle, probe)
    t_seq = (time.perf_counter() - t0) / 4
    total = max(1, args.steps + args.warmup)
    nseq = int(max(1, min(cfg["batch"], round(60.0 / (total * max(t_seq, 1e-4))))))
    inp = cpu_inputs(np, cfg, nseq)
    for _ in range(args.warmup):
        cpu_scan_layer(oracle, inp)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_scan_layer(oracle, inp)
    dt = time.perf_counter() - t0
    elems = args.steps * nseq * L * D * N
    value = elems / dt
    sample = (f"each step: one layer's scan fwd+bwd on {nseq} of the {cfg['batch']} sequences "
              f"({nseq * L * D * N} elements); fp32 oracle/scan_oracle.c, OpenMP")
    workload = (f"{cfg['layers']}-layer momentum-Mamba scan fwd+bwd (expand 2, d_state {N}): "
                f"B={cfg['batch']} L={L} D={D} N={N} per layer, softplus(delta+bias) and SiLU(z) "
                f"gate fused, fp32")
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / max(1, args.steps),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": workload, "batch": cfg["batch"], "seqlen": L, "dim": D,
                   "dstate": N, "layers": cfg["layers"], "beta": BETA, "alpha": ALPHA,
                   "parallelism": "host cores (rank 0 only)"},
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


def run_long(ctx, steps):
    """B=8, L=65536, D=2048, N=16 with bf16 activations, fp32 state: the
    sequence is split into WORLD_SIZE contiguous segments, one per rank
    (segment summaries all-gathered over NCCL, carries folded locally).  Total
    work is fixed (strong scaling)."""
    import torch
    import torch.distributed as dist

    from momentummamba_b200.selective_scan import ScanCall
    from momentummamba_b200.seqshard import SegmentOps as ops

    args = ctx.args
    world, rank, dev = ctx.world, ctx.rank, ctx.dev
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
    ms, clocks = timed_region(ctx, step, steps)
    phases = None
    if args.phases and marks:
        names = ["start", "fwd_carry", "fwd", "bwd_carry", "bwd"]
        phases = {}
        for a, b in zip(names[:-1], names[1:]):
            t = statistics.mean(marks[a][i].elapsed_time(marks[b][i]) for i in range(steps))
            phases[b] = ctx_max(t, ctx)
    del x, delta, Bm, Cm, dout, call
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    elems = Bsz * L * D * N
    fb, bb = long_bytes(Bsz, Lr, D, N)
    peak, peak_kind = load_peaks()
    ms_step = ms / steps
    achieved = (fb + bb) / (ms_step / 1e3) / 1e9  # per GPU: its segment's bytes over the step
    return {
        "metric": METRIC, "value": elems / (ms_step / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms_step,
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
        "gpu_launches": (3 if world == 1 else 6) * steps,
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------
# LinOSS layer scan workload (IM and IMEX discretisations)
# ---------------------------------------------------------------------------
LINOSS = dict(batch=16, seqlen=4096, osc=256)


def run_linoss(ctx, steps):
    """The LinOSS layer scan (LinOSS_pytorch.py:153-239, time-invariant 2x2
    transition built in-kernel) forward + backward for IM and IMEX at B=16
    L=4096 P=256 with complex Bu ~ N(0,1), A ~ U[0,1], step = exp(U[ln 1e-3,
    ln 1e-1]).  One step = IM fwd + bwd and IMEX fwd + bwd; elements = B L P
    oscillator steps per discretisation.  Batch-sharded over ranks (weak)."""
    import torch

    from momentummamba_b200 import _lib

    args, dev, world = ctx.args, ctx.dev, ctx.world
    lib = _lib.load()
    Bsz, L, P = LINOSS["batch"], LINOSS["seqlen"], LINOSS["osc"]
    g = torch.Generator(device=dev).manual_seed(5 + ctx.rank)
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
    graph = capture(ctx, stepfn)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ms, clocks = timed_region(ctx, graph.replay, steps)
    t = launch_times((("fwd_IM", lambda: fwd(0)), ("bwd_IM", lambda: bwd(0)),
                      ("fwd_IMEX", lambda: fwd(1)), ("bwd_IMEX", lambda: bwd(1))))
    del graph, Bu, dx2, x2, dBu, works
    torch.cuda.empty_cache()
    if ctx.rank != 0:
        return None
    elems = Bsz * L * P
    fwd_b = elems * 16 + 2 * P * 4          # read Bu, write x2 (complex fp32)
    bwd_b = elems * 24 + 4 * P * 4          # read Bu, dx2; write dBu
    peak, peak_kind = load_peaks()
    achieved = bwd_b / (t["bwd_IM"] / 1e3) / 1e9
    tr = load_traffic("linoss_bwd_traffic.json")
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = linoss_cpu_baseline(budget_s=min(5.0, args.cpu_budget))
    return {
        "metric": METRIC, "value": job_rate(2 * elems * steps, world, ms), "unit": UNIT,
        "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
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
        "gpu_launches": 14 * steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }


def run_linoss_layer(ctx, steps):
    """The whole LinOSSLayer (LinOSS_pytorch.py:258-312) forward + backward, IM and
    IMEX, at H=128 P=256 B=16 L=4096: Bu = B u and y = Re(C x2) + D u with their
    gradients on the tensor cores (tcgen05, 3 x tf32) around the LinOSS scan
    kernels.  Beside it, the same layer with the contractions as fp32 cuBLAS
    GEMMs (torch.matmul; the reference's einsums) around the same scan.
    Elements = B L P oscillator steps per discretisation."""
    import torch

    import momentummamba_b200.LinOSS_pytorch as lp
    from momentummamba_b200.scan2 import linoss_scan

    args, dev, world = ctx.args, ctx.dev, ctx.world
    Bsz, L, P, H = LINOSS["batch"], LINOSS["seqlen"], LINOSS["osc"], 128
    torch.manual_seed(11 + ctx.rank)
    layers = [lp.LinOSSLayer(P, H, d).to(dev) for d in ("IM", "IMEX")]
    u = torch.randn(Bsz, L, H, device=dev, requires_grad=True)
    gy = torch.randn(Bsz, L, H, device=dev)

    def cublas_layer(layer, x):
        A = torch.relu(layer.A_diag)
        s = torch.sigmoid(layer.steps)
        bu = torch.complex(x @ layer.B_real.t(), x @ layer.B_imag.t())
        x2 = linoss_scan(layer.discretization, A, s, bu)
        return x2.real @ layer.C_real.t() - x2.imag @ layer.C_imag.t() + x * layer.D

    def step_tc():
        for ly in layers:
            ly(u).backward(gy)

    def step_cublas():
        for ly in layers:
            cublas_layer(ly, u).backward(gy)

    for _ in range(max(3, args.warmup)):
        step_tc()
        step_cublas()
    torch.cuda.synchronize()
    ms, clocks = timed_region(ctx, step_tc, steps)
    ms_cu, _ = timed_region(ctx, step_cublas, max(3, steps // 4))
    ms_cu *= steps / max(3, steps // 4)
    # one of the four tensor-core GEMM shapes alone: Bu = u Bm^T (M = B L, N = 2P, K = H)
    from momentummamba_b200.tc_gemm import gemm_nt, split_tf32
    u2 = u.detach().reshape(Bsz * L, H)
    Bm = split_tf32(torch.randn(2 * P, H, device=dev))   # as the layer: weights split once
    t = launch_times((("tc_gemm Bu", lambda: gemm_nt(u2, Bm)),))
    del layers, u, gy, u2, Bm
    torch.cuda.empty_cache()
    if ctx.rank != 0:
        return None
    elems = Bsz * L * P
    peak, peak_kind = load_peaks()
    gemm_b = Bsz * L * (H + 2 * P) * 4            # read u, write Bu
    achieved = gemm_b / (t["tc_gemm Bu"] / 1e3) / 1e9
    return {
        "metric": METRIC, "value": job_rate(2 * elems * steps, world, ms), "unit": UNIT,
        "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "LinOSSLayer forward + backward (GEMMs + scan), IM and IMEX: "
                               "B=16 L=4096 H=128 P=256, u ~ N(0,1), module init",
                   "parallelism": f"batch-sharded x{world}", "launch": "eager (autograd)",
                   "l2": "inputs larger than L2 (Bu, x2 134 MB each)"},
        "cublas_contractions_ms_per_step": ms_cu / steps,
        "roofline": {"kernel": "tc_gemm_ws_kernel (Bu = u Bm^T, M=65536 N=512 K=128, "
                               "weights split once)",
                     "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s", "frac": achieved / peak,
                     "algorithmic_bytes": gemm_b, "ms_per_launch": t["tc_gemm Bu"],
                     "traffic": None},
        # per discretisation: forward 2 GEMMs + 3 scan launches, backward 4 GEMMs + 4
        "gpu_launches": 26 * steps,
        "clocks": clocks,
    }


def linoss_cpu_baseline(budget_s=5.0):
    """The fp32 oracle's 2x2 scan (forward + backward) on the host cores, for one
    sequence of the LinOSS workload (IM transition)."""
    import numpy as np

    import oracle
    cores = cpu_threads()
    oracle.set_num_threads(cores)
    L, P = LINOSS["seqlen"], LINOSS["osc"]
    rng = np.random.default_rng(0)
    Ad = rng.uniform(0, 1, P)
    st = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), P))
    S = 1.0 / (1.0 + st ** 2 * Ad)
    M = np.broadcast_to(np.concatenate([1.0 - st ** 2 * Ad * S, -st * Ad * S, st * S, S]),
                        (1, L, 4 * P)).astype(np.float32)
    Fc = (rng.standard_normal((1, L, 2 * P)) + 1j * rng.standard_normal((1, L, 2 * P))).astype(
        np.complex64)
    gX = (rng.standard_normal((1, L, 2 * P)) + 1j * rng.standard_normal((1, L, 2 * P))).astype(
        np.complex64)
    t0 = time.perf_counter()
    n = 0
    while True:
        Ms, X = oracle.scan2_fwd(M, Fc, prec="f32")
        oracle.scan2_bwd(M, X, gX, prec="f32")
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": n * L * P / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} fwd+bwd passes of the generic 2x2 scan over 1 of the 16 sequences "
                      f"(L={L}, P={P}, complex F), {dt:.1f} s; fp32 oracle/scan_oracle.c"}


# ---------------------------------------------------------------------------
# row-form and PScan-layout scans (the reference's materialised-tensor paths)
# ---------------------------------------------------------------------------
def run_rows(ctx, steps):
    """The momentum row scan (momentum_scan_cuda.py:204-253: R = B*D*N rows of L
    steps) and the diagonal scan in the PScan layout (pscan.py:43-234: (B, L,
    D*N)) forward + backward at the d_model-128 stack's size (B=32, L=1024,
    D=256, N=16: 134,217,728 elements each).  One step = rows fwd + bwd, then
    pscan fwd + bwd; elements = the rows scan's (the line's value), per-kernel
    GB/s for both.  Batch-sharded replicas over ranks (weak)."""
    import torch

    from momentummamba_b200 import _lib

    args, dev, world = ctx.args, ctx.dev, ctx.world
    lib = _lib.load()
    BS, L, D, N = STACK1["batch"], STACK1["seqlen"], STACK1["dim"], STACK1["dstate"]
    R, M = BS * D * N, D * N
    g = torch.Generator(device=dev).manual_seed(7 + ctx.rank)
    a = torch.exp(-torch.rand(R, L, device=dev, generator=g) * 0.2)     # decay factors in (0.82, 1]
    u = torch.randn(R, L, device=dev, generator=g)
    gr = torch.randn(R, L, device=dev, generator=g)
    h, da, du = torch.empty_like(a), torch.empty_like(a), torch.empty_like(a)
    A3, X3, G3 = a.view(BS, L, M), u.view(BS, L, M), gr.view(BS, L, M)  # same bytes, PScan layout
    H3, dA3, dX3 = torch.empty_like(A3), torch.empty_like(A3), torch.empty_like(A3)
    Pp = _lib.ptr

    def rows_fwd():
        _lib.check(lib.mmb_rows_fwd(R, L, Pp(a), BETA, Pp(u), Pp(h), None, _lib.stream_of(a)),
                   "rows fwd")

    def rows_bwd():
        _lib.check(lib.mmb_rows_bwd(R, L, Pp(gr), Pp(a), BETA, Pp(h), Pp(da), Pp(du),
                                    _lib.stream_of(a)), "rows bwd")

    def ps_fwd():
        _lib.check(lib.mmb_pscan_fwd(BS, L, M, Pp(A3), Pp(X3), Pp(H3), _lib.stream_of(a)),
                   "pscan fwd")

    def ps_bwd():
        _lib.check(lib.mmb_pscan_bwd(BS, L, M, Pp(A3), Pp(H3), Pp(G3), Pp(dA3), Pp(dX3),
                                     _lib.stream_of(a)), "pscan bwd")

    def stepfn():
        rows_fwd()
        rows_bwd()
        ps_fwd()
        ps_bwd()

    for _ in range(max(3, args.warmup)):
        stepfn()
    torch.cuda.synchronize()
    graph = capture(ctx, stepfn)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ms, clocks = timed_region(ctx, graph.replay, steps)
    t = launch_times((("rows_fwd", rows_fwd), ("rows_bwd", rows_bwd), ("pscan_fwd", ps_fwd),
                      ("pscan_bwd", ps_bwd)))
    del graph, a, u, gr, h, da, du, H3, dA3, dX3
    torch.cuda.empty_cache()
    if ctx.rank != 0:
        return None
    elems = R * L
    nbytes = {"rows_fwd": 12 * elems, "rows_bwd": 20 * elems,   # a, u -> h; g, a, h -> da, du
              "pscan_fwd": 12 * elems, "pscan_bwd": 20 * elems}  # A, X -> H; A, H, G -> dA, dX
    peak, peak_kind = load_peaks()
    kern = {k: {"ms": v, "algorithmic_bytes": nbytes[k], "GB/s": nbytes[k] / (v / 1e3) / 1e9,
                "frac": nbytes[k] / (v / 1e3) / 1e9 / peak} for k, v in t.items()}
    return {
        "metric": METRIC, "value": job_rate(elems * steps, world, ms), "unit": UNIT,
        "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "materialised-tensor scans at the d_model-128 stack's size: "
                               "momentum row scan (R=131072 rows x L=1024, beta 0.6) and "
                               "PScan-layout diagonal scan (B=32 L=1024 M=4096), fwd+bwd each; "
                               "value = row-scan elements/s over the whole step",
                   "parallelism": f"batch-sharded x{world}", "launch": "cuda graph",
                   "l2": "inputs larger than L2 (537 MB per tensor)"},
        "roofline": {"kernel": "rows_bwd", "bound": "hbm", "achieved": kern["rows_bwd"]["GB/s"],
                     "peak": peak, "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s",
                     "frac": kern["rows_bwd"]["frac"], "algorithmic_bytes": nbytes["rows_bwd"],
                     "ms_per_launch": t["rows_bwd"], "traffic": None},
        "kernels": kern,
        "gpu_launches": 4 * steps,
        "clocks": clocks,
    }


def summary(line):
    """The part of a workload's line kept as an extra key of the default line."""
    if line is None:
        return None
    keep = ("value", "unit", "n_gpus", "steps", "ms_per_step", "scaling", "dtype", "config",
            "roofline", "kernels", "time_chunks", "unsplit", "cublas_contractions_ms_per_step",
            "phases_ms", "gpu_launches", "clocks", "cpu_baseline")
    return {k: line[k] for k in keep if k in line}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="default workload only (no extra keys)")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--workload", choices=["classifier", "stack", "chunks", "long", "linoss",
                                           "linoss_layer", "rows"],
                    default="classifier",
                    help="classifier: the 6-layer momentum-Mamba classifier scan, B=256 T=300 "
                         "D=512 split over the ranks (the benchmark line, with the other "
                         "workloads as extra keys); stack: the 4-layer d_model-128 stack, "
                         "B=32 L=1024 D=256 per rank; chunks: 4 layers of B=2 L=8192 D=256 "
                         "split along time inside the GPU; long: B=8 L=65536 D=2048 bf16, "
                         "sequence-sharded; linoss: the LinOSS layer scan, IM and IMEX, "
                         "B=16 L=4096 P=256; rows: the row-form and PScan-layout scans")
    ap.add_argument("--kernels-only", action="store_true",
                    help="classifier/stack: warm-up and steps as eager launches, nothing "
                         "else (for profiler captures)")
    ap.add_argument("--batch", type=int, default=0,
                    help="classifier/stack: sequences per rank (profiling of a smaller case "
                         "only; the benchmark line uses the configuration's batch)")
    ap.add_argument("--phases", action="store_true",
                    help="long workload: also time each phase (adds events to the step)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    ctx = Ctx(args)
    ctx.init_gpu()
    K = args.steps
    if args.workload == "classifier":
        line = run_stack(ctx, CLASSIFIER, True, K, with_e2e=True, with_cpu=True,
                         name="classifier")
        if not args.no_extras and not args.kernels_only:
            extras = {}
            if ctx.world == 1:
                extras["stack_cfg1"] = summary(run_stack(ctx, STACK1, False, 4 * K,
                                                         with_e2e=False, with_cpu=True,
                                                         name="stack_cfg1"))
            extras["long_seq"] = summary(run_long(ctx, max(3, K // 40)))
            if ctx.world == 1:
                extras["time_chunks"] = summary(run_stack(ctx, CHUNKED, False, K,
                                                          with_e2e=False, with_cpu=False,
                                                          name="time_chunks"))
                extras["linoss"] = summary(run_linoss(ctx, 2 * K))
                extras["linoss_layer"] = summary(run_linoss_layer(ctx, max(3, K // 4)))
                extras["rows"] = summary(run_rows(ctx, max(3, K // 4)))
            if line is not None:
                line["extras"] = extras
                line["gpu_launches_extras"] = sum(
                    (v or {}).get("gpu_launches", 0) for v in extras.values())
    elif args.workload == "stack":
        line = run_stack(ctx, STACK1, False, K, with_e2e=True, with_cpu=True, name="stack_cfg1")
    elif args.workload == "chunks":
        line = run_stack(ctx, CHUNKED, False, K, with_e2e=False, with_cpu=False,
                         name="time_chunks")
    elif args.workload == "long":
        line = run_long(ctx, K)
    elif args.workload == "linoss":
        line = run_linoss(ctx, K)
    elif args.workload == "linoss_layer":
        line = run_linoss_layer(ctx, K)
    else:
        line = run_rows(ctx, K)
    ctx.close()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
