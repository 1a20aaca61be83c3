#!/usr/bin/env python
"""Benchmark: Hyena FFT-conv fwd+bwd throughput (GElem/s, E = B*C*N) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg1|cfg2|cfg3|cfg0] [--impl b200|reference]

One "step" = forward + backward of the fused Hyena mixer (configs 1-3: short depthwise
conv, gates, FFT long conv with D-skip) or of the op-level causal conv (config 0) on one
batch of seeded synthetic input. Inputs are resident in HBM for ``value``; ``e2e`` runs
the same step through the public API from pinned host buffers: the H2D copy of every
input and the D2H copy of the step's output y are inside the timed region (the next
step's inputs are copied on a second stream while the current step computes, as a
training loop prefetches its next batch), while the gradients stay on the device (where
an optimizer step would read them).

Default workload: config 2 (B=8, C=256, 128x128, bf16). On one GPU the run also measures
config 1 (the ViT grid) the same way and reports it under ``secondary``.

Multi-GPU (torchrun, one rank per GPU): config 2 shards the batch (strong scaling: B=8
split over the ranks), and every timed step ends with one NCCL all-reduce of the filter,
D and short-conv gradients (partial sums over each rank's images); config 3 shards the
channels (no collective); config 1 runs one independent replica per rank (weak
scaling). The time is the max over ranks of the device-timed region.

``--impl reference`` times the reference's CPU path (the CPU oracle restating
nvsubquadratic/ops/fftconv.py + hyena_nd.py on torch.fft) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "Hyena FFT-conv fwd+bwd GElem/s (B·C·N) at 1/2/4/8 B200; % of HBM roofline"

CONFIGS = {
    # name: dict(nd, B, C, S, K, short, gates, dtype, causal, shard)
    "cfg0": dict(nd=1, B=2, C=64, S=(4096,), K=(4096,), short=0, g1="identity", g2="identity",
                 dtype=torch.float32, causal=True, shard="replica", op_only=True,
                 desc="1D causal FFT long conv + D skip, fp32 (reference CPU case)"),
    "cfg1": dict(nd=2, B=32, C=768, S=(14, 14), K=(14, 14), short=3, g1="identity", g2="identity",
                 dtype=torch.bfloat16, causal=False, shard="replica",
                 desc="2D HyenaND ViT-B grid 14x14, SIREN-style 14x14 filter, F=24x24 (linear-conv length 21 padded to 3*2^3), 3x3 short conv"),
    "cfg2": dict(nd=2, B=8, C=256, S=(128, 128), K=(128, 128), short=3, g1="identity", g2="identity",
                 dtype=torch.bfloat16, causal=False, shard="batch",
                 desc="2D HyenaND 128x128, exp-radial 128x128 filter, F=192x192 (alias-free for N=128, K=128), batch-sharded"),
    "cfg3": dict(nd=3, B=2, C=192, S=(64, 64, 64), K=(64, 64, 64), short=3, g1="identity", g2="identity",
                 dtype=torch.bfloat16, causal=False, shard="channel",
                 desc="3D HyenaND 64^3, full-extent exp-radial filter, F=128^3, channel-sharded"),
    "cfg4": dict(nd=1, B=1, C=4096, S=(1 << 20,), K=(1 << 20,), short=7, g1="identity", g2="identity",
                 dtype=torch.bfloat16, causal=True, shard="cp",
                 desc="1D causal long-context Hyena, L=2^20, context-parallel (zigzag sequence shards, "
                      "NCCL all-to-all to channel shards and back), F=2^21, causal short conv k=7"),
}


# ----------------------------------------------------------------- inputs
def siren_filter(C: int, K: tuple[int, ...], gen: torch.Generator, hidden: int = 32, omega0: float = 30.0):
    """Random-init SIREN-style MLP evaluated on a [-1, 1]^d grid of K points: [1, C, *K] fp32.
    (Filter generation is not part of the hot path; this only makes a realistic filter.)"""
    nd = len(K)
    axes = [torch.linspace(-1.0, 1.0, k) for k in K]
    grid = torch.stack(torch.meshgrid(*axes, indexing="ij"), dim=-1).reshape(-1, nd)
    W1 = (torch.rand(nd, hidden, generator=gen) * 2 - 1) / nd
    W2 = (torch.rand(hidden, hidden, generator=gen) * 2 - 1) * math.sqrt(6 / hidden) / omega0
    W3 = (torch.rand(hidden, C, generator=gen) * 2 - 1) * math.sqrt(6 / hidden) / omega0
    h = torch.sin(omega0 * grid @ W1)
    h = torch.sin(omega0 * h @ W2)
    out = h @ W3
    return out.t().reshape((1, C) + tuple(K)).contiguous() * 0.1


def decay_filter(C: int, K: tuple[int, ...], gen: torch.Generator, causal: bool):
    """N(0,1) * exp(-beta_c * r): radius from the filter centre (or time for causal 1D)."""
    nd = len(K)
    if causal:
        r = torch.arange(K[0], dtype=torch.float32).view(1, -1)
        beta = (torch.rand(C, 1, generator=gen) * 4.5 + 0.5) / K[0]
    else:
        axes = [torch.arange(k, dtype=torch.float32) - (k - 1) / 2 for k in K]
        mesh = torch.stack(torch.meshgrid(*axes, indexing="ij"), dim=0)
        r = mesh.pow(2).sum(0).sqrt().reshape(1, -1)
        beta = (torch.rand(C, 1, generator=gen) * 4.5 + 0.5) / max(K)
    f = torch.randn((C, r.shape[1]), generator=gen) * torch.exp(-beta * r)
    f = f / math.sqrt(r.shape[1])
    return f.reshape((1, C) + tuple(K))


def make_inputs(cfg: dict, B: int, C: int, c_off: int, seed: int = 0):
    """Seeded synthetic inputs on the CPU (activations, filter, D, short-conv weights, dy in that order)."""
    g = torch.Generator().manual_seed(seed)
    nd, S, K, dt = cfg["nd"], cfg["S"], cfg["K"], cfg["dtype"]
    if cfg.get("op_only"):
        x = torch.randn((B, C) + S, generator=g)
        filt = decay_filter(C, K, g, causal=True)
        D = torch.randn(C, generator=g)
        dy = torch.randn((B, C) + S, generator=g)
        return dict(x=x.to(dt), filt=filt, D=D.to(dt), dy=dy.to(dt))
    qkv = torch.randn((B,) + S + (3 * C,), generator=g).to(dt)
    if S == (14, 14):
        filt = siren_filter(C, K, g)
    else:
        filt = decay_filter(C, K, g, causal=cfg["causal"])
    D = ((torch.rand(C, generator=g) * 2 - 1) / math.sqrt(C)).to(dt)
    sk = cfg["short"]
    sw = ((torch.rand((3 * C, 1) + (sk,) * nd, generator=g) * 2 - 1) / math.sqrt(sk ** nd)).to(dt) if sk else None
    dy = torch.randn((B,) + S + (C,), generator=g).to(dt)
    return dict(qkv=qkv, filt=filt, D=D, sw=sw, dy=dy)


def alg_bytes(cfg: dict, B: int, C: int) -> int:
    """Minimum HBM bytes of one fwd+bwd (nothing kept between passes but the inputs)."""
    N = math.prod(cfg["S"])
    E = B * C * N
    KK = math.prod(cfg["K"])
    if cfg.get("op_only"):
        return 20 * E + 12 * C * KK  # fp32: x, y, dy, x, dx + filter read x2, dfilt write
    s = torch.finfo(cfg["dtype"]).bits // 8
    # fwd: read q,k,v, write y; bwd: read dy, q,k,v, write dq,dk,dv; filter read twice + dfilt
    return (11 * s) * E + 12 * C * KK


# ----------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.rows: list[list[str]] = []
        self._stop = threading.Event()
        self._proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 10 and self._proc.poll() is None:
                time.sleep(0.02)  # wait for the first sample before the caller starts timing
        except (OSError, FileNotFoundError):
            self._proc = None
        return self

    def _read(self):
        for line in self._proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()

    def summary(self):
        rows = [r for r in self.rows if len(r) >= 7 and r[0].isdigit()]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [int(r[0]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][1]), "reasons": reasons,
                "samples": len(rows)}


# ----------------------------------------------------------------- CPU reference arm
def cpu_reference_time(cfg: dict, budget_s: float = 20.0):
    """Time the reference's CPU path (oracle restatement on torch.fft) on a channel slice
    of the workload; returns (GElem/s, threads, sample description)."""
    from oracle.fftconv import fftconv_bhl
    from oracle.hyena import hyena_forward

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    B, C = cfg["B"], cfg["C"]
    N = math.prod(cfg["S"])
    # pick a channel slice that takes ~1 s per fwd+bwd (grown from a tiny probe)
    c_s = max(1, min(C, 8))

    def one(cs):
        inp = make_inputs(cfg, B if cfg["nd"] < 3 else min(B, 2), cs, 0, seed=0)
        t0 = time.perf_counter()
        if cfg.get("op_only"):
            x = inp["x"].requires_grad_(True)
            k = inp["filt"].requires_grad_(True)
            D = inp["D"].requires_grad_(True)
            y = fftconv_bhl(x, k, D, causal=True)
            y.backward(inp["dy"])
        else:
            q, k, v = (t.clone().requires_grad_(True) for t in inp["qkv"].chunk(3, dim=-1))
            f = inp["filt"].requires_grad_(True)
            D = inp["D"].clone().requires_grad_(True)
            sw = inp["sw"].clone().requires_grad_(True) if inp["sw"] is not None else None
            y = hyena_forward(q, k, v, f, D, sw, None, causal=cfg["causal"], gate1=cfg["g1"], gate2=cfg["g2"])
            y.backward(inp["dy"])
        return time.perf_counter() - t0

    one(c_s)  # warm-up (first-call allocation / thread-pool start-up)
    t = one(c_s)
    while t < 1.0 and c_s < C:
        c_s = min(C, c_s * 2)
        t = one(c_s)
    reps = max(3, min(15, int(budget_s / max(t, 1e-3))))
    times = [one(c_s) for _ in range(reps)]
    med = statistics.median(times)
    Bs = B if cfg["nd"] < 3 else min(B, 2)
    elems = Bs * c_s * N
    sample = f"{Bs}x{c_s} of {B}x{C} (batch x channels), full spatial extent; median of {reps} fwd+bwd"
    return elems / med / 1e9, threads, sample, med


# ----------------------------------------------------------------- per-pass timing
def pass_bytes(cfg: dict, B: int, C: int) -> dict:
    """Algorithmic HBM bytes of each library pass (they sum to alg_bytes)."""
    E = B * C * math.prod(cfg["S"])
    KK = math.prod(cfg["K"])
    if cfg.get("op_only"):
        return {"hyfft_conv_forward": 8 * E + 4 * C * KK, "hyfft_conv_backward": 12 * E + 8 * C * KK}
    s = torch.finfo(cfg["dtype"]).bits // 8
    return {"hyfft_hyena_forward": 4 * s * E + 4 * C * KK, "hyfft_hyena_backward": 7 * s * E + 8 * C * KK}


def time_passes(step, zero_grads, flush, names, n):
    """Mean device time of each named C-ABI call over n eager steps, CUDA events recorded
    on the stream the library launches on (torch's current stream), L2 flushed right
    before every timed call."""
    from nvsubquadratic_b200 import _lib

    lib = _lib.load()
    recs = {nm: [] for nm in names}
    origs = {nm: getattr(lib, nm) for nm in names}

    def wrap(nm, orig):
        def timed(*a):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            rc = orig(*a)
            e.record()
            recs[nm].append((s, e))
            return rc
        return timed

    try:
        for nm, orig in origs.items():
            setattr(lib, nm, wrap(nm, orig))
        for _ in range(n):
            zero_grads()
            step()
        torch.cuda.synchronize()
    finally:
        for nm, orig in origs.items():
            setattr(lib, nm, orig)
    return {nm: sum(a.elapsed_time(b) for a, b in r) / len(r) for nm, r in recs.items() if r}


# ----------------------------------------------------------------- context-parallel arm
def run_cp(args, cfg, rank, world, device):
    """cfg4: every rank holds its zigzag sequence chunks of q, k, v (one [B, L/P, 3C]
    projection output) and its channel block of the filter; a step is the CP mixer's
    forward + backward (two NCCL all-to-alls each way). Eager steps (the collectives stay
    outside CUDA graphs); inputs are far larger than L2, so no flush is needed."""
    from types import SimpleNamespace

    from nvsubquadratic_b200 import _lib, cp

    group = torch.distributed.group.WORLD
    B, C, L = cfg["B"], cfg["C"], cfg["S"][0]
    P = world
    assert C % P == 0 and L % (2 * P) == 0
    d, l = C // P, L // P
    dt = cfg["dtype"]
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    qkv = torch.randn((B, l, 3 * C), generator=gen, device=device, dtype=dt).requires_grad_(True)
    dy = torch.randn((B, l, C), generator=gen, device=device, dtype=dt)
    gc = torch.Generator(device=device).manual_seed(7)  # identical parameters on every rank
    t = torch.arange(L, device=device, dtype=torch.float32)
    alpha = (torch.rand(C, generator=gc, device=device) * 4.5 + 0.5) / L
    filt = torch.randn((1, d, L), generator=gen, device=device) * torch.exp(-alpha[rank * d:(rank + 1) * d, None] * t)
    filt.requires_grad_(True)
    del t
    D = ((torch.rand(C, generator=gc, device=device) * 2 - 1) / math.sqrt(C)).requires_grad_(True)
    sk = cfg["short"]
    sw = ((torch.rand((3 * C, 1, sk), generator=gc, device=device) * 2 - 1) / math.sqrt(sk)).requires_grad_(True)
    mod = SimpleNamespace(shortcut=D, short_weight=sw, short_bias=None, causal=True, short_causal=True,
                          gate1=cfg["g1"], gate2=cfg["g2"])
    params = [qkv, filt, D, sw]

    def zero_grads():
        for p_ in params:
            p_.grad = None

    def step():
        q, k, v = qkv.chunk(3, dim=-1)
        y = cp.hyena_context_parallel(mod, q, k, v, filt, group)
        y.backward(dy)
        return y

    for _ in range(args.warmup):
        zero_grads()
        step()
    torch.cuda.synchronize()
    if args.profile:
        return None
    n0 = _lib.launch_count()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        # the timed steps start together on every rank (the sampler's start-up differs per rank)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            zero_grads()
            starts[i].record()
            step()
            ends[i].record()
        torch.cuda.synchronize()
    torch.distributed.barrier()
    launches = (_lib.launch_count() - n0) // max(1, args.steps)
    total_ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
    tt = torch.tensor([total_ms], device=device)
    torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
    total_ms = tt.item()
    # the dominant library pass on the local channel block
    names = ["hyfft_hyena_forward", "hyfft_hyena_backward"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    pass_ms = time_passes(step, zero_grads, flush, names, 1)
    for nm in names:
        t3 = torch.tensor([pass_ms[nm]], device=device)
        torch.distributed.all_reduce(t3, op=torch.distributed.ReduceOp.MAX)
        pass_ms[nm] = t3.item()
    # e2e: local inputs from pinned host memory, outputs and gradients back, per step
    host_qkv = torch.empty(qkv.shape, dtype=qkv.dtype, pin_memory=True)
    host_qkv.copy_(qkv.detach())
    host_dy = torch.empty(dy.shape, dtype=dy.dtype, pin_memory=True)
    host_dy.copy_(dy)
    outs = None
    e2e = []
    for i in range(2):
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.distributed.barrier()
        a.record()
        x = host_qkv.to(device, non_blocking=True).requires_grad_(True)
        g_ = host_dy.to(device, non_blocking=True)
        filt.grad = None
        q, k, v = x.chunk(3, dim=-1)
        y = cp.hyena_context_parallel(mod, q, k, v, filt, group)
        y.backward(g_)
        res = [y]  # the step's result; gradients stay on the device for the optimizer
        if outs is None:
            outs = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
        for o, r in zip(outs, res):
            o.copy_(r, non_blocking=True)
        b_.record()
        torch.cuda.synchronize()
        e2e.append(a.elapsed_time(b_))
        del x, g_, y, res, q, k, v
    te = torch.tensor([min(e2e)], device=device)
    torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
    h2d = host_qkv.numel() * host_qkv.element_size() + host_dy.numel() * host_dy.element_size()
    d2h = sum(o.numel() * o.element_size() for o in outs)
    return dict(pass_ms=pass_ms, total_ms=total_ms, launches=launches, clocks=clk.summary(), B=B, C=d,
                e2e_ms=te.item(), h2d=h2d, d2h=d2h)


# ----------------------------------------------------------------- GPU arm
def run_gpu(args, cfg, rank, world, device):
    from nvsubquadratic_b200 import _lib
    from nvsubquadratic_b200.fftconv import causal_fftconv1d_fp32_bhl
    from nvsubquadratic_b200.hyena import hyena_fused

    from nvsubquadratic_b200.dp import GradBucket, batch_shard

    B, C = cfg["B"], cfg["C"]
    c_off = 0
    if world > 1 and cfg["shard"] == "batch":
        # the full batch's seeded inputs, this rank's slice of the activations
        inp = make_inputs(cfg, B, C, 0, seed=0)
        for key in ("qkv", "dy", "x"):
            if key in inp:
                inp[key] = batch_shard(inp[key], rank, world).contiguous()
        B //= world
    else:
        if world > 1 and cfg["shard"] == "channel":
            assert C % world == 0
            C //= world
            c_off = rank * C
        inp = make_inputs(cfg, B, C, c_off, seed=rank if cfg["shard"] == "replica" else 0)
    dev_inp = {k: (v.to(device) if v is not None else None) for k, v in inp.items()}
    # batch shards: the parameter gradients are partial sums over the rank's batch slice;
    # one NCCL all-reduce of a flat fp32 bucket (filter, D, short-conv) completes each step
    dp_group = torch.distributed.group.WORLD if (world > 1 and cfg["shard"] == "batch") else None

    op_only = cfg.get("op_only", False)
    if op_only:
        x = dev_inp["x"].requires_grad_(True)
        filt = dev_inp["filt"].requires_grad_(True)
        D = dev_inp["D"].requires_grad_(True)
        dy = dev_inp["dy"]

        def step():
            y = causal_fftconv1d_fp32_bhl(x, filt, D)
            y.backward(dy)
            return y

        params = [x, filt, D]
    else:
        qkv = dev_inp["qkv"].requires_grad_(True)
        filt = dev_inp["filt"].requires_grad_(True)
        D = dev_inp["D"].requires_grad_(True)
        sw = dev_inp["sw"].requires_grad_(True) if dev_inp["sw"] is not None else None
        dy = dev_inp["dy"]

        def step():
            q, k, v = qkv.chunk(3, dim=-1)
            y = hyena_fused(q, k, v, filt, D, sw, None, causal=cfg["causal"], gate1=cfg["g1"], gate2=cfg["g2"])
            y.backward(dy)
            return y

        params = [p for p in (qkv, filt, D, sw) if p is not None]

    def zero_grads():
        for p in params:
            p.grad = None

    bucket = GradBucket([p for p in params if p is not (x if op_only else qkv)], device) if dp_group else None

    def reduce_grads():
        if bucket is not None:
            bucket.reduce(dp_group)

    # eager warm-up (also counts kernel launches of one step)
    for _ in range(max(1, args.warmup)):
        zero_grads()
        step()
        reduce_grads()
    torch.cuda.synchronize()
    if args.profile:
        for _ in range(args.steps):
            zero_grads()
            step()
            reduce_grads()
        torch.cuda.synchronize()
        return None
    n0 = _lib.launch_count()
    zero_grads()
    step()
    torch.cuda.synchronize()
    launches_per_step = _lib.launch_count() - n0

    # capture one step in a CUDA graph (the hot loop is launch-bound otherwise)
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for _ in range(2):
            zero_grads()
            step()
    torch.cuda.current_stream(device).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    zero_grads()
    with torch.cuda.graph(graph):
        step()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # > 126 MB L2
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # estimate the step time to size an untimed, clock-sampled burn-in of ~0.5 s right before
    # the timed steps (nvidia-smi samples every 50 ms; a short timed region alone gets 0-1 samples);
    # every rank runs the same number of burn-in steps (the slowest rank's estimate)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    est = torch.tensor([max(e0.elapsed_time(e1) / 3, 1e-3)], device=device)
    if world > 1:
        torch.distributed.all_reduce(est, op=torch.distributed.ReduceOp.MAX)
    n_burn = int(min(20000, max(10, 500.0 / est.item())))
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        for _ in range(n_burn):
            graph.replay()
        # the timed steps start together on every rank: barrier + synchronize right before them
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()  # evict L2 between timed steps (outside the events)
            starts[i].record()
            graph.replay()
            reduce_grads()  # batch shards: gradient all-reduce inside the timed step
            ends[i].record()
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    step_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    total_ms = t.item()

    del graph
    names = list(pass_bytes(cfg, B, C))
    pass_ms = time_passes(step, zero_grads, flush, names, max(3, min(args.steps, 10)))
    for nm in names:
        t3 = torch.tensor([pass_ms[nm]], device=device)
        if world > 1:
            torch.distributed.all_reduce(t3, op=torch.distributed.ReduceOp.MAX)
        pass_ms[nm] = t3.item()

    # e2e through the public API from pinned host buffers (eager, no graph)
    e2e_ms, h2d, d2h, copy_ms = e2e_time(cfg, inp, device, op_only, max(3, min(args.steps, 10)), dp_group)
    t2 = torch.tensor([e2e_ms], device=device)
    if world > 1:
        torch.distributed.all_reduce(t2, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = t2.item()
    return dict(pass_ms=pass_ms, total_ms=total_ms, step_ms=step_ms, launches=launches_per_step, clocks=clk.summary(),
                B=B, C=C, e2e_ms=e2e_ms, h2d=h2d, d2h=d2h, copy_ms=copy_ms)


def e2e_time(cfg, inp, device, op_only, steps, dp_group=None):
    """End-to-end steps through the public API from pinned host buffers.

    Every step copies all of its inputs (activations, upstream gradient and the parameters)
    host -> device, runs forward + backward through hyena_fused / the op API, and copies its
    result y device -> host. The copies of step i + 1 run on a copy stream while step i
    computes (two device slots per input), the way a training loop prefetches its next
    batch; the time of a block of steps is the device span from its first copy to its last
    device -> host copy, divided by the number of steps, and the median of three blocks is
    reported. Returns (ms per step, H2D
    bytes per step, D2H bytes per step, ms of one step's H2D copies alone)."""
    from nvsubquadratic_b200.dp import GradBucket
    from nvsubquadratic_b200.fftconv import causal_fftconv1d_fp32_bhl
    from nvsubquadratic_b200.hyena import hyena_fused

    names = ["x", "filt", "D", "dy"] if op_only else ["qkv", "filt", "D", "sw", "dy"]
    host = {k: inp[k].pin_memory() for k in names if inp.get(k) is not None}
    # the host->device copies alone (same pinned buffers), to separate link time from the rest
    copy_times = []
    for _ in range(5):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        _tmp = [t.to(device, non_blocking=True) for t in host.values()]
        b.record()
        torch.cuda.synchronize()
        copy_times.append(a.elapsed_time(b))
        del _tmp
    main = torch.cuda.current_stream(device)
    cs = torch.cuda.Stream(device)
    slots = [{k: torch.empty(v.shape, dtype=v.dtype, device=device) for k, v in host.items()} for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    for e in freed:
        e.record(main)
    out = None

    def issue_copy(i):
        s = i % 2
        with torch.cuda.stream(cs):
            cs.wait_event(freed[s])  # step i - 2 is done with this slot
            for k, v in host.items():
                slots[s][k].copy_(v, non_blocking=True)
            copied[s].record(cs)

    def run_step(i):
        nonlocal out
        s = i % 2
        main.wait_event(copied[s])
        d = {k: v.detach().requires_grad_(k != "dy") for k, v in slots[s].items()}
        if op_only:
            y = causal_fftconv1d_fp32_bhl(d["x"], d["filt"], d["D"])
        else:
            q, k, v = d["qkv"].chunk(3, dim=-1)
            y = hyena_fused(q, k, v, d["filt"], d["D"], d.get("sw"), None, causal=cfg["causal"], gate1=cfg["g1"],
                            gate2=cfg["g2"])
        y.backward(d["dy"])
        if dp_group is not None:  # batch shards: full-batch parameter gradients
            GradBucket([d["filt"], d["D"], d.get("sw")], device).reduce(dp_group)
        if out is None:
            out = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        out.copy_(y, non_blocking=True)  # the step's result; gradients stay on the device
        freed[s].record(main)
        return y

    n_warm = 3
    issue_copy(0)
    for i in range(n_warm):
        if i + 1 < n_warm:
            issue_copy(i + 1)
        run_step(i)
    torch.cuda.synchronize()
    # timed: blocks of exactly `steps` copies in, `steps` fwd+bwd, `steps` copies out; three
    # blocks, the median block reported (one host-side stall of the eager path, an allocator
    # or scheduler hiccup, must not stand for the path)
    blocks = []
    base = n_warm
    for _ in range(3):
        if dp_group is not None:  # the ranks start each timed block together
            torch.distributed.barrier(group=dp_group)
            torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(main)
        issue_copy(base)
        for i in range(steps):
            if i + 1 < steps:
                issue_copy(base + i + 1)
            run_step(base + i)
        t1.record(main)
        torch.cuda.synchronize()
        blocks.append(t0.elapsed_time(t1) / steps)
        base += steps
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out.numel() * out.element_size()
    return statistics.median(blocks), h2d, d2h, statistics.median(copy_times[1:])


def measure_filter_gen(device, steps: int, warmup: int) -> dict:
    """The implicit filter generator (SIREN network + exponential window, forward and backward:
    nvsubquadratic_b200.siren.ckconv_filter) on the reference's double grid of cfg1 (27x27
    points, 768 channels) and of cfg2 (255x255 points, 256 channels), 3 SIREN layers of width
    64, embedding 32: device time per fwd+bwd (CUDA events, median), filter values per second,
    and the CPU oracle (torch, all host threads) on the cfg1 case."""
    from nvsubquadratic_b200.siren import SIRENKernelB200, ckconv_filter
    from oracle import siren as osr

    res = {"layers": 3, "hidden": 64, "embedding": 32, "stat": "median of the timed fwd+bwd calls"}
    for name, C, seq in (("cfg1", 768, (14, 14)), ("cfg2", 256, (128, 128))):
        torch.manual_seed(0)
        m = SIRENKernelB200(out_dim=C, data_dim=2, mlp_hidden_dim=64, num_layers=3, embedding_dim=32, omega_0=10.0,
                            L_cache=seq[0], use_bias=True).to(device)
        mw = osr.mask_init(2, C).to(device)
        G = (2 * seq[0] - 1) * (2 * seq[1] - 1)
        dk = torch.randn(1, C, 2 * seq[0] - 1, 2 * seq[1] - 1, device=device)
        times = []
        for i in range(warmup + steps):
            m.zero_grad(set_to_none=True)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            ckconv_filter(m, mw, seq, layout="bhl").backward(dk)
            e1.record()
            torch.cuda.synchronize()
            if i >= warmup:
                times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
        res[name] = {"grid": [2 * seq[0] - 1, 2 * seq[1] - 1], "channels": C, "ms_fwd_bwd": round(ms, 4),
                     "gvalues_per_s": round(G * C / (ms * 1e-3) / 1e9, 3)}
        if name == "cfg1":
            cpu = {k: v.detach().cpu() for k, v in m.state_dict().items()}
            p = {"pe.weight": cpu["positional_embedding.linear.weight"], "pe.bias": cpu["positional_embedding.linear.bias"],
                 "out.weight": cpu["out_linear.weight"], "out.bias": cpu["out_linear.bias"]}
            for i in range(2):
                p[f"hidden.{i}.weight"] = cpu[f"hidden_linears.{i}.weight"]
                p[f"hidden.{i}.bias"] = cpu[f"hidden_linears.{i}.bias"]
            p = {k: v.requires_grad_(True) for k, v in p.items()}
            mwc, dkc = mw.cpu(), dk.cpu().permute(0, 2, 3, 1)
            ct = []
            for _ in range(3):
                t0 = time.perf_counter()
                osr.siren_filter(p, seq, seq[0], mwc)[0].backward(dkc)
                ct.append(time.perf_counter() - t0)
            res[name]["cpu_oracle_ms"] = round(statistics.median(ct) * 1e3, 3)
            res[name]["cpu_threads"] = torch.get_num_threads()
    return res


def summarize(name: str, cfg: dict, res: dict, world: int, steps: int, peaks: dict) -> dict:
    """Whole-job throughput (all ranks' elements / max-over-ranks time), the roofline of the
    dominant library pass and the end-to-end throughput of one measured configuration."""
    N = math.prod(cfg["S"])
    elems_job = res["B"] * res["C"] * N * world
    t_step = res["total_ms"] / steps / 1e3
    peak = peaks.get("hbm_gbs", 6650.0)
    step_achieved = alg_bytes(cfg, res["B"], res["C"]) / t_step / 1e9
    pbytes = pass_bytes(cfg, res["B"], res["C"])
    dom = max(res["pass_ms"], key=res["pass_ms"].get)
    achieved = pbytes[dom] / (res["pass_ms"][dom] / 1e3) / 1e9
    traffic = None
    if world == 1:  # the captures are of the single-GPU workload
        try:
            with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
                traffic = json.load(f).get(name, {}).get(dom)
        except (OSError, ValueError):
            pass
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "kernel": dom, "pass_ms": {k: round(v, 4) for k, v in res["pass_ms"].items()},
                "pass_bytes": pbytes,
                "scope": "dominant library pass: its algorithmic bytes / its mean CUDA-event time "
                         "(L2 flushed before each timed call); traffic = ncu dram read+write bytes "
                         "per call from profiles/ncu_traffic.json",
                "step_achieved": round(step_achieved, 1), "step_frac": round(step_achieved / peak, 4),
                "peak_source": ("MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks
                                else "fallback 6650 GB/s (of fallback)")}
    return {"value": elems_job / t_step / 1e9, "t_step": t_step, "roofline": roofline,
            "e2e_value": elems_job / (res["e2e_ms"] / 1e3) / 1e9}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--secondary", default="cfg1",
                    help="on one GPU, also measure this configuration and report it under 'secondary' ('' for none)")
    ap.add_argument("--filter-gen", default=True, action=argparse.BooleanOptionalAction,
                    help="on one GPU, also time the implicit filter generator (SIREN + window, fwd+bwd)")
    ap.add_argument("--profile", action="store_true",
                    help="run warmup + steps eager fwd+bwd steps and exit (for ncu captures)")
    ap.add_argument("--channels", type=int, default=None,
                    help="with --profile: run the config's shapes with this many channels (a smaller device "
                         "footprint for full ncu captures; the kernels and line lengths are the config's own)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    if args.channels is not None:
        if not args.profile:
            raise SystemExit("--channels only applies to --profile runs (bench lines use the config as published)")
        cfg = dict(cfg, C=args.channels)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    B, C = cfg["B"], cfg["C"]
    N = math.prod(cfg["S"])
    dtname = {torch.float32: "f32", torch.bfloat16: "bf16"}[cfg["dtype"]]
    config = {"workload": args.config + ": " + cfg["desc"], "batch": B, "channels": C, "spatial": list(cfg["S"]),
              "filter": list(cfg["K"]), "sharding": cfg["shard"], "l2": "flushed between timed steps (256 MB write)"}
    if cfg["shard"] == "batch":
        config["parallelism"] = (f"dp{world}: batch shards of {B // world if B % world == 0 else '?'} images per "
                                 "rank, filter/D/short-conv gradients summed by one NCCL all-reduce of a flat fp32 "
                                 "bucket inside every timed step" if world > 1 else "dp1")
    if cfg["shard"] == "cp":
        config["l2"] = "inputs (GBs per rank) far larger than L2; no flush"
        config["parallelism"] = f"cp{world}"
        # keep the engine's spectrum workspace (and the filter-spectrum cache, kept only where
        # it fits this budget: P >= 4) small next to the 1M-long activations
        os.environ.setdefault("HYFFT_WS_BUDGET_MB", "4096")
        # GB-sized activations of varying shapes: avoid caching-allocator fragmentation
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

    if args.impl == "reference":
        if rank != 0:
            return
        gel, threads, sample, med = cpu_reference_time(cfg)
        out = {"metric": METRIC, "value": round(gel, 6), "unit": "GElem/s", "n_gpus": args.gpus, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3), "higher_is_better": True,
               "scaling": "weak" if cfg["shard"] == "replica" else "strong", "vs_baseline": None, "dtype": dtname,
               "data": "synthetic", "config": config, "impl": "reference",
               "cpu_baseline": {"value": round(gel, 6), "unit": "GElem/s", "cores": threads, "kind": "port",
                                "sample": sample},
               "e2e": {"value": round(gel, 6), "unit": "GElem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(out))
        return

    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if cfg["shard"] == "cp" and world == 1 and args.profile:
        # one GPU, --profile: the mixer on one channel block at full length (what every rank
        # runs between the exchanges), for kernel captures
        res = run_gpu(args, dict(cfg, shard="replica"), rank, world, device)
    elif cfg["shard"] == "cp":
        if world < 2:
            raise SystemExit("cfg4 (context parallel, 12.9 GB of q/k/v per copy) runs on 2 or more GPUs "
                             "(python -m torch.distributed.run ... bench.py --config cfg4 --gpus N); "
                             "on one GPU only as --profile --channels C (the local channel block)")
        res = run_cp(args, cfg, rank, world, device)
    else:
        res = run_gpu(args, cfg, rank, world, device)
    if res is None:  # --profile
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    summ = summarize(args.config, cfg, res, world, args.steps, peaks)
    value, t_step, e2e_val = summ["value"], summ["t_step"], summ["e2e_value"]

    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 4), "unit": "GElem/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_step * 1e3, 4), "higher_is_better": True,
            "scaling": "weak" if cfg["shard"] == "replica" else "strong", "vs_baseline": None, "dtype": dtname,
            "data": "synthetic (seeded N(0,1) activations, random-init filters)", "config": config,
            "roofline": summ["roofline"],
            "e2e": {"value": round(e2e_val, 4), "unit": "GElem/s", "h2d_bytes_per_step": res["h2d"],
                    "d2h_bytes_per_step": res["d2h"], "ms_per_step": round(res["e2e_ms"], 4),
                    "h2d_copy_ms": round(res["copy_ms"], 4) if res.get("copy_ms") is not None else None,
                    "stat": "median of three blocks of timed steps, each block's mean per step (eager, through "
                            "hyena_fused / the op API); every step's inputs copied H2D from pinned memory and y "
                            "copied D2H, the next step's H2D overlapped with this step's compute on a copy stream"},
            "gpu_launches": res["launches"] * args.steps,
            "clocks": res["clocks"],
        }
        if world == 1 and not args.no_cpu_baseline:
            gel, threads, sample, _ = cpu_reference_time(cfg)
            out["cpu_baseline"] = {"value": round(gel, 6), "unit": "GElem/s", "cores": threads, "kind": "port",
                                   "sample": sample}
        if world == 1 and args.secondary and args.secondary != args.config:
            # a second configuration measured the same way in the same run (single GPU only)
            cfg2 = CONFIGS[args.secondary]
            res2 = run_gpu(args, cfg2, rank, world, device)
            s2 = summarize(args.secondary, cfg2, res2, world, args.steps, peaks)
            out["secondary"] = {"workload": args.secondary + ": " + cfg2["desc"], "value": round(s2["value"], 4),
                                "unit": "GElem/s", "ms_per_step": round(s2["t_step"] * 1e3, 4),
                                "roofline": s2["roofline"],
                                "e2e": {"value": round(s2["e2e_value"], 4), "unit": "GElem/s",
                                        "ms_per_step": round(res2["e2e_ms"], 4), "h2d_bytes_per_step": res2["h2d"],
                                        "d2h_bytes_per_step": res2["d2h"]},
                                "gpu_launches": res2["launches"] * args.steps, "clocks": res2["clocks"]}
        if world == 1 and args.filter_gen:
            out["filter_gen"] = measure_filter_gen(device, args.steps, args.warmup)
        print(json.dumps(out))
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
