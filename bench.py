"""Headline benchmark: post_attn_mlp at Llama-3-8B widths on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode step's MLP half: 32 stacked post_attn_mlp layers
(hidden 4096, intermediate 14336, bf16, independent seeded weights), replayed
as one CUDA graph.  The metric is microseconds per layer at M=1 (M=8 is
reported beside it) and the HBM bandwidth that implies, against the measured
copy roof.  With N>1 GPUs (torchrun) the same 32-layer stack runs tensor-
parallel: gate/up column-sharded, down row-sharded, one partial-sum exchange
per layer -- over the NVLink exchange buffers by default, NCCL all_reduce with
--tp-collective nccl (strong scaling: the total work is fixed).

Rank 0 prints ONE JSON line.  --impl reference times the reference's CPU
formulation of the same layer (the oracle port of reference.py, numpy fp32) on
the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I = 4096, 14336
LAYERS = 32
EPS = 1e-5
PUBLISHED_US = {1: 1570.0, 8: 1621.0}  # reference bf16 post_attn_mlp, RTX 4070 Laptop
METRIC = "post_attn_mlp us/layer at M=1 (Llama-3-8B widths, 32-layer CUDA graph), HBM GB/s vs measured peak"


def layer_bytes(m: int, h: int = H, i: int = I, world: int = 1) -> int:
    """Algorithmic HBM bytes of one layer on one rank: weights once, hidden in,
    out, norm weight.  Intermediates stay in L2 and are not counted."""
    return (2 * i * h + h * i) * 2 // world + 2 * m * h * 2 + h * 2 if m else 0


def gate_up_launch_bytes(m: int, world: int = 1) -> int:
    """Algorithmic bytes of one gate/up-kernel launch: weight, hidden, norm weight, mid."""
    return 2 * I * H * 2 // world + m * H * 2 + H * 2 + m * (I // world) * 2


def down_launch_bytes(m: int, world: int = 1) -> int:
    """Algorithmic bytes of one down-kernel launch: weight, mid, residual, output."""
    return H * I * 2 // world + m * (I // world) * 2 + 2 * m * H * 2


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def committed_traffic() -> dict:
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.lines: list[tuple[float, str]] = []
        self.proc = None
        self.thread = None
        self.window = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        time.sleep(0.3)

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def mark(self, t0: float, t1: float) -> None:
        """Restrict the summary to samples taken in [t0, t1] (the timed region)."""
        self.window = (t0, t1)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = self.lines
        if self.window is not None:
            inside = [ln for t, ln in lines if self.window[0] <= t <= self.window[1] + 0.15]
            lines = inside if inside else [ln for _, ln in lines]
        else:
            lines = [ln for _, ln in lines]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU leg
def cpu_layer_sample(layers: int, m: int, seed: int = 0):
    """Seeded fp32 copies (bf16-rounded values) of `layers` Llama-3-8B MLP layers for the CPU leg."""
    from oracle import fd_oracle as O

    rng = np.random.default_rng(seed)
    out = []
    for _ in range(layers):
        nw = O.round_bf16(1 + 0.1 * rng.standard_normal(H, dtype=np.float32))
        wgu = O.round_bf16(rng.standard_normal((2 * I, H), dtype=np.float32) * np.float32(0.02))
        wd = O.round_bf16(rng.standard_normal((H, I), dtype=np.float32) * np.float32(0.02))
        out.append((nw, wgu, wd))
    x = O.round_bf16(rng.standard_normal((m, H), dtype=np.float32))
    return x, out


def cpu_time_layers(x, layers, budget_s: float, min_evals: int, max_evals: int | None = None):
    """Time the oracle's post_attn_mlp per layer; returns (us/layer, evals, threads)."""
    from oracle import fd_oracle as O

    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(os.cpu_count())
        threads = max((d.get("num_threads", 1) for d in threadpool_info()), default=1)
    except Exception:  # threadpoolctl missing: BLAS picks its own count
        threads = os.cpu_count()
    times = []
    t_end = time.perf_counter() + budget_s
    j = 0
    while (len(times) < min_evals or time.perf_counter() < t_end) and (max_evals is None or len(times) < max_evals):
        nw, wgu, wd = layers[j % len(layers)]
        t0 = time.perf_counter()
        x = O.post_attn_mlp(x, nw, wgu, wd, EPS, O.BF16)
        times.append(time.perf_counter() - t0)
        j += 1
    return statistics.median(times) * 1e6, len(times), threads


def workload_config(m: int, world: int, collective: str) -> dict:
    """The `config` object both arms print: the workload the metric is quoted on."""
    return {
        "workload": f"post_attn_mlp Llama-3-8B widths, M={m}, {LAYERS} layers in one CUDA graph"
                    + (f", tensor-parallel x{world} ({collective} partial-sum exchange per layer)" if world > 1 else ""),
        "hidden": H, "intermediate": I, "m": m, "layers": LAYERS, "kind": "dot",
        "parallelism": f"tp{world}" if world > 1 else "single",
        "l2": f"inputs larger than L2: {LAYERS * layer_bytes(m, world=world) / 1e9:.1f} GB of weights per step per GPU",
    }


def run_reference(args) -> None:
    """The reference arm: the reference's CPU formulation (oracle port) on host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    m = args.m
    x, layers = cpu_layer_sample(2, m)
    cpu_time_layers(x, layers, 0.0, max(1, args.warmup), max(1, args.warmup))  # warm-up
    us, evals, threads = cpu_time_layers(x, layers, 0.0, args.steps, args.steps)
    sample = (f"{evals} single-layer steps over 2 seeded Llama-3-8B MLP layers, M={m}, numpy fp32 "
              f"(oracle port of reference.py:66-79) on the host cores; each step is one layer of the workload")
    line = {
        "impl": "reference", "metric": METRIC, "value": us, "unit": "us/layer",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": us / 1e3,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights rounded to bf16)",
        "config": workload_config(m, args.gpus, args.tp_collective),
        "cpu_baseline": {"value": us, "unit": "us/layer", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": us, "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU legs
def make_layers(torch, device, layers, world=1, rank=0, dtype=None):
    """Seeded layers (seed = layer index): norm_w = 1 + 0.1 N(0,1), weights N(0, 0.02).

    With world > 1 each rank keeps only its tensor-parallel shard.
    """
    from fused_decode_b200 import tp

    dtype = dtype or torch.bfloat16
    out = []
    for layer in range(layers):
        g = torch.Generator(device=device)
        g.manual_seed(layer)
        nw = (1 + 0.1 * torch.randn(H, device=device, generator=g)).to(dtype)
        wgu = torch.empty(2 * I, H, device=device, dtype=dtype)
        wd = torch.empty(H, I, device=device, dtype=dtype)
        # generate in chunks to bound the fp32 temporary
        for r0 in range(0, 2 * I, 4096):
            wgu[r0:r0 + 4096] = (torch.randn(min(4096, 2 * I - r0), H, device=device, generator=g) * 0.02).to(dtype)
        for r0 in range(0, H, 1024):
            wd[r0:r0 + 1024] = (torch.randn(min(1024, H - r0), I, device=device, generator=g) * 0.02).to(dtype)
        if world > 1:
            wgu, wd = tp.shard_gate_up(wgu, rank, world), tp.shard_down(wd, rank, world)
        out.append((nw, wgu, wd))
    return out


def cuda_time(torch, fn, iters: int) -> float:
    """Average ms per call of fn() over iters, CUDA events on the current stream."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def copy_roof_gbs(torch, device) -> float:
    from fused_decode_b200 import kernels as K

    n = 1 << 29  # 1 GiB of bf16 per buffer
    a = torch.empty(n, device=device, dtype=torch.bfloat16).normal_()
    b = torch.empty_like(a)
    for _ in range(3):
        K.launch_copy(b, a)
    ms = cuda_time(torch, lambda: K.launch_copy(b, a), 10)
    del a, b
    return 2 * n * 2 / (ms * 1e-3) / 1e9


L2_BYTES = 126 * 1024 * 1024
GEMV_SHAPES = ((4096, 4096), (14336, 4096), (4096, 14336), (28672, 4096))
GEMV_MS = (1, 2, 4, 8, 16)


def graph_time_us(torch, calls, reps: int = 3, inner: int = 20) -> float:
    """Device time per call (us) of a rotation of `calls` replayed in a CUDA
    graph of `inner` calls; median of `reps` timed replays after 3 warm-up."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for c in calls:
            c()
    torch.cuda.current_stream().wait_stream(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for j in range(inner):
            calls[j % len(calls)]()
    for _ in range(3):
        g.replay()
    times = [cuda_time(torch, g.replay, 1) for _ in range(reps)]
    del g
    return statistics.median(times) * 1e3 / inner


def copies_for(nbytes: int) -> int:
    """Input copies to rotate so one pass touches at least 2x L2."""
    return max(1, -(-2 * L2_BYTES // max(nbytes, 1)))


def run_ops(torch, device, roof_gbs: float, peak_gbs: float) -> dict:
    """Standalone ops at the BASELINE shapes: us per call, algorithmic GB/s and
    fractions of the in-process copy roof and of the measured peak."""
    import fused_decode_b200 as fd

    g = torch.Generator(device=device).manual_seed(0)
    out: dict = {}

    def rec(name, us, nbytes, **extra):
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"us": us, "bytes": nbytes, "gbs": gbs, "frac_copy_roof": gbs / roof_gbs,
                     "frac_peak": gbs / peak_gbs, **extra}

    f16 = torch.float16
    # add+RMSNorm and RMSNorm
    for rows in (8192, 1):
        w = (1 + 0.1 * torch.randn(H, device=device, generator=g)).to(f16)
        n_add = 4 * rows * H * 2 + H * 2
        k = copies_for(n_add)
        xs = [torch.randn(rows, H, device=device, dtype=f16, generator=g) for _ in range(k)]
        rs = [torch.randn(rows, H, device=device, dtype=f16, generator=g) for _ in range(k)]
        os_ = [torch.empty(rows, H, device=device, dtype=f16) for _ in range(k)]
        calls = [(lambda j=j: fd.add_rms_norm(xs[j], rs[j], w, 1e-5, out=os_[j], residual_out=rs[j]))
                 for j in range(k)]
        rec(f"add_rms_norm_{rows}x{H}_f16", graph_time_us(torch, calls), n_add)
        n_rms = 2 * rows * H * 2 + H * 2
        calls = [(lambda j=j: fd.rms_norm(xs[j], w, 1e-5, out=os_[j])) for j in range(k)]
        rec(f"rms_norm_{rows}x{H}_f16", graph_time_us(torch, calls), n_rms)
        del xs, rs, os_
    # SwiGLU (config 1)
    for rows in (2048, 1):
        for dt, tag in ((f16, "f16"), (torch.bfloat16, "bf16")):
            nb = 3 * rows * I * 2
            k = copies_for(nb)
            gs = [torch.randn(rows, I, device=device, dtype=dt, generator=g) for _ in range(k)]
            us_ = [torch.randn(rows, I, device=device, dtype=dt, generator=g) for _ in range(k)]
            os_ = [torch.empty(rows, I, device=device, dtype=dt) for _ in range(k)]
            calls = [(lambda j=j: fd.swiglu(gs[j], us_[j], out=os_[j])) for j in range(k)]
            rec(f"swiglu_{rows}x{I}_{tag}", graph_time_us(torch, calls), nb)
            del gs, us_, os_
    # RoPE (config 1): x [1, T, 32, 128], cos/sin [T, 1, 128] from theta = 500000
    for t in (2048, 1):
        cos, sin = rope_tables(torch, t, 128, device, f16)
        nb = 2 * t * 32 * 128 * 2 + 2 * t * 128 * 2
        k = copies_for(nb)
        xs = [torch.randn(1, t, 32, 128, device=device, dtype=f16, generator=g) for _ in range(k)]
        os_ = [torch.empty_like(xs[0]) for _ in range(k)]
        calls = [(lambda j=j: fd.rope(xs[j], cos, sin, out=os_[j])) for j in range(k)]
        rec(f"rope_1x{t}x32x128_f16", graph_time_us(torch, calls), nb)
        del xs, os_
    # linear_decode sweep (config 2); weights rotate through >= 2x L2
    for dt, tag in ((torch.bfloat16, "bf16"), (f16, "f16")):
        for n, kk in GEMV_SHAPES:
            k = copies_for(n * kk * 2)
            ws = [(torch.randn(n, kk, device=device, generator=g) * 0.02).to(dt) for _ in range(k)]
            for m in GEMV_MS:
                x = torch.randn(m, kk, device=device, dtype=dt, generator=g)
                y = torch.empty(m, n, device=device, dtype=dt)
                calls = [(lambda j=j: fd.linear_decode(x, ws[j], out=y, kind="dot")) for j in range(k)]
                nb = (m * kk + n * kk + m * n) * 2
                rec(f"linear_decode_m{m}_n{n}_k{kk}_{tag}", graph_time_us(torch, calls), nb)
            if n == 4096 and kk == 14336:  # the down projection with bias + row_add
                for m in (1, 8):
                    x = torch.randn(m, kk, device=device, dtype=dt, generator=g)
                    b = (torch.randn(n, device=device, generator=g) * 0.02).to(dt)
                    ra = torch.randn(m, n, device=device, dtype=dt, generator=g)
                    y = torch.empty(m, n, device=device, dtype=dt)
                    calls = [(lambda j=j: fd.linear_decode(x, ws[j], b, row_add=ra, out=y, kind="dot"))
                             for j in range(k)]
                    nb = (m * kk + n * kk + 2 * m * n + n) * 2
                    rec(f"linear_decode_m{m}_n{n}_k{kk}_{tag}_bias_rowadd", graph_time_us(torch, calls), nb)
            del ws
    torch.cuda.empty_cache()
    return out


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from fused_decode_b200 import _capi, post_attn_mlp, tp
    from fused_decode_b200 import kernels as K
    from fused_decode_b200.stack import MlpStack

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    _capi.load()
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    pk = peaks()
    layers = make_layers(torch, device, LAYERS, world, rank)

    exchange = None
    if world > 1 and args.tp_collective == "nvlink":
        exchange = tp.TPExchange(H, m_max=16)

    def layer_fn_tp(x, nw, wgu, wd):
        return tp.TPPostAttnMlp(nw, wgu, wd, EPS, kind="dot", exchange=exchange)(x)

    def build_stack(m):
        fn = layer_fn_tp if world > 1 else None
        return MlpStack(layers, m, EPS, kind="dot", layer_fn=fn)

    def time_stack(stack, steps, warmup, sampler=None):
        x0 = torch.randn(stack.static_in.shape, device=device, dtype=torch.bfloat16,
                         generator=torch.Generator(device=device).manual_seed(1234))
        stack.static_in.copy_(x0)
        for _ in range(warmup):
            stack.replay()
        if sampler:
            sampler.start()  # before the barrier: every rank starts its clock together
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        s.record()
        for _ in range(steps):
            stack.replay()
        e.record()
        torch.cuda.synchronize()
        if sampler:
            sampler.mark(t0, time.perf_counter())
        clocks = sampler.stop() if sampler else None
        barrier()
        return max_over_ranks(s.elapsed_time(e) / steps), clocks

    # ---- headline: M=1 stack
    roof = copy_roof_gbs(torch, device) if rank == 0 else None
    stack1 = build_stack(args.m)
    sampler = ClockSampler(local) if rank == 0 else None
    ms1, clocks = time_stack(stack1, args.steps, args.warmup, sampler)
    us1 = ms1 * 1e3 / LAYERS
    bytes1 = layer_bytes(args.m, world=world)
    # ---- M=8 beside it
    stack8 = build_stack(8)
    ms8, _ = time_stack(stack8, args.steps, args.warmup)
    us8 = ms8 * 1e3 / LAYERS
    bytes8 = layer_bytes(8, world=world)

    # ---- the same stack as one launch per layer (the per-call public API)
    per_layer_us = None
    if world == 1:
        stack_pl = MlpStack(layers, args.m, EPS, kind="dot", fused=False)
        ms_pl, _ = time_stack(stack_pl, max(3, args.steps // 5), args.warmup)
        per_layer_us = ms_pl * 1e3 / LAYERS
        del stack_pl

    # ---- the same stack as two stream-K kernels per layer (gate/up, then down + residual)
    two_kernel_us = None
    if world == 1:
        hb = [torch.zeros(args.m, H, device=device, dtype=torch.bfloat16) for _ in range(3)]
        mid2 = torch.empty(args.m, I, device=device, dtype=torch.bfloat16)

        def two_kernel_all():
            x = hb[0]
            for li, (nw, wgu, wd) in enumerate(layers):
                K.mlp_gate_up_out(x, nw, wgu, mid2, EPS, "dot")
                y = hb[1 + (li & 1)]
                K.linear_out(mid2, wd, y, row_add=x, kind="dot")
                x = y

        two_kernel_all()
        t_stream = torch.cuda.Stream()
        t_stream.wait_stream(torch.cuda.current_stream())
        graph_tk = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_tk, stream=t_stream):
            two_kernel_all()
        for _ in range(args.warmup):
            graph_tk.replay()
        two_kernel_us = cuda_time(torch, graph_tk.replay, max(3, args.steps // 5)) * 1e3 / LAYERS
        del graph_tk

    # ---- the gate/up stage alone (its own kernel), 32 launches per graph
    mid = torch.empty(args.m, I // world, device=device, dtype=torch.bfloat16)
    xk = torch.randn(args.m, H, device=device, dtype=torch.bfloat16)

    def gate_up_all():
        for nw, wgu, _ in layers:
            K.mlp_gate_up_out(xk, nw, wgu, mid, EPS, "dot")

    gate_up_all()
    g_stream = torch.cuda.Stream()
    g_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(g_stream):
        gate_up_all()
    torch.cuda.current_stream().wait_stream(g_stream)
    graph_gu = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_gu, stream=g_stream):
        gate_up_all()
    for _ in range(args.warmup):
        graph_gu.replay()
    ms_gu = max_over_ranks(cuda_time(torch, graph_gu.replay, max(3, args.steps // 5))) / LAYERS
    gu_bytes = gate_up_launch_bytes(args.m, world)
    gu_gbs = gu_bytes / (ms_gu * 1e-3) / 1e9

    # ---- the down stage alone (+ residual), 32 launches per graph
    yd = torch.empty(args.m, H, device=device, dtype=torch.bfloat16)
    mid_d = torch.randn(args.m, I // world, device=device, dtype=torch.bfloat16)

    def down_all():
        for _, _, wd in layers:
            K.linear_out(mid_d, wd, yd, row_add=xk, kind="dot")

    down_all()
    d_stream = torch.cuda.Stream()
    d_stream.wait_stream(torch.cuda.current_stream())
    graph_dn = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_dn, stream=d_stream):
        down_all()
    for _ in range(args.warmup):
        graph_dn.replay()
    ms_dn = max_over_ranks(cuda_time(torch, graph_dn.replay, max(3, args.steps // 5))) / LAYERS
    dn_bytes = down_launch_bytes(args.m, world)
    dn_gbs = dn_bytes / (ms_dn * 1e-3) / 1e9

    # ---- e2e: public API with host buffers, every step H2D + 32 layers + D2H
    host_in = torch.randn(args.m, H, dtype=torch.bfloat16).pin_memory()
    host_out = torch.empty(args.m, H, dtype=torch.bfloat16).pin_memory()

    def e2e_graph_step():
        out = stack1(host_in)  # H2D copy into the graph's input, replay
        host_out.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def e2e_eager_step():
        x = host_in.to(device, non_blocking=True)
        for nw, wgu, wd in layers:
            x = layer_fn_tp(x, nw, wgu, wd) if world > 1 else post_attn_mlp(x, nw, wgu, wd, EPS, kind="dot")
        host_out.copy_(x, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def wall(fn, steps):
        for _ in range(args.warmup):
            fn()
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            fn()
        dt = (time.perf_counter() - t0) / steps
        barrier()
        return max_over_ranks(dt)

    e2e_s = wall(e2e_graph_step, args.steps)
    e2e_eager_s = wall(e2e_eager_step, max(3, args.steps // 10))

    # ---- CPU baseline (rank 0, N=1 only): oracle port, bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        xs, cl = cpu_layer_sample(2, args.m)
        cpu_time_layers(xs, cl, 0.0, 1, 1)
        us_cpu, evals, threads = cpu_time_layers(xs, cl, args.cpu_seconds, 3)
        cpu = {"value": us_cpu, "unit": "us/layer", "cores": threads, "kind": "port",
               "sample": f"{evals} layer evaluations over 2 seeded Llama-3-8B MLP layers at M={args.m} "
                         f"(numpy fp32 oracle port of reference.py:66-79), ~{args.cpu_seconds:.0f} s"}

    ops = None
    if world == 1 and not args.no_ops:
        ops = run_ops(torch, device, roof, pk["hbm_gbs"])

    if rank == 0:
        traffic = committed_traffic().get(f"gate_up_kernel_bytes_per_launch_m{args.m}") if world == 1 else None
        gbs1 = bytes1 / (us1 * 1e-6) / 1e9
        line = {
            "metric": METRIC,
            "value": us1,
            "unit": "us/layer",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms1,
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": us1 / PUBLISHED_US[1] if args.m == 1 else None,
            "dtype": "bf16",
            "data": "synthetic (seeded random-init Llama-3-8B MLP weights, N(0,0.02))",
            "config": workload_config(args.m, world, args.tp_collective),
            "hbm_gbs": gbs1,
            "hbm_frac": gbs1 / pk["hbm_gbs"],
            "copy_roof_gbs": roof,
            "m8": {"us_per_layer": us8, "ms_per_step": ms8, "hbm_gbs": bytes8 / (us8 * 1e-6) / 1e9,
                   "hbm_frac": bytes8 / (us8 * 1e-6) / 1e9 / pk["hbm_gbs"]},
            # the dominant kernel: RMSNorm + gate/up GEMV + SwiGLU (2/3 of a layer's bytes)
            "roofline": {
                "kernel": "gemv_tma_kernel<bf16, GATEUP> (RMSNorm prologue + gate/up GEMV + SwiGLU epilogue)",
                "bound": "hbm", "achieved": gu_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": gu_gbs / pk["hbm_gbs"], "peak_source": pk["source"],
                "traffic": traffic, "bytes_per_launch": gu_bytes, "us_per_launch": ms_gu * 1e3,
                "timed": "32 launches (one per layer's weights) in one CUDA graph, CUDA events",
            },
            "kernels": {
                "gate_up_stage_alone": {"us": ms_gu * 1e3, "gbs": gu_gbs, "bytes": gu_bytes,
                                        "frac": gu_gbs / pk["hbm_gbs"]},
                "down_stage_alone": {"us": ms_dn * 1e3, "gbs": dn_gbs, "bytes": dn_bytes,
                                     "frac": dn_gbs / pk["hbm_gbs"]},
                "layer": {"us": us1, "gbs": gbs1, "bytes": bytes1, "frac": gbs1 / pk["hbm_gbs"]},
                "per_layer_calls_us_per_layer": per_layer_us,
                "two_kernel_us_per_layer": two_kernel_us,
            },
            "ops": ops,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_s * 1e6 / LAYERS, "unit": "us/layer",
                    "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
                    "d2h_bytes_per_step": host_out.numel() * host_out.element_size(),
                    "api": "fused_decode_b200.stack.MlpStack (pinned host in, graph replay, pinned host out)",
                    "eager_api_us_per_layer": e2e_eager_s * 1e6 / LAYERS},
            # single GPU: two launches per layer; tensor-parallel: gate/up, down
            # and reduce (NVLink exchange) or residual-add (after NCCL) per layer
            "gpu_launches": args.steps * (stack1.launches_per_replay if world == 1 else 3 * LAYERS),
            "tp_collective": args.tp_collective if world > 1 else None,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        del stack1, stack8, graph_gu, graph_dn
        torch.cuda.synchronize()
        if exchange is not None:
            exchange.close()
        dist.destroy_process_group()


NCU_CASES = ("gate_up", "down", "mlp", "add_rms", "rms", "swiglu", "rope", "copy")


def run_ncu_case(args) -> None:
    """A small fixed workload for an ncu capture: 2 warm-up launches, then 3
    launches of the named kernel (one layer, Llama-3-8B widths, M = --m).
    Prints nothing but a one-line summary; never used for timing."""
    import torch

    import fused_decode_b200 as fd
    from fused_decode_b200 import _capi
    from fused_decode_b200 import kernels as K

    _capi.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    m, bf = args.m, torch.bfloat16
    case = args.ncu_case
    if case in ("gate_up", "down", "mlp"):
        (nw, wgu, wd), = make_layers(torch, dev, 1)
        x = torch.randn(m, H, device=dev, dtype=bf, generator=g)
        mid = torch.randn(m, I, device=dev, dtype=bf, generator=g)
        y = torch.empty(m, H, device=dev, dtype=bf)
        fn = {
            "gate_up": lambda: K.mlp_gate_up_out(x, nw, wgu, mid, EPS, "dot"),
            "down": lambda: K.linear_out(mid, wd, y, row_add=x, kind="dot"),
            "mlp": lambda: fd.post_attn_mlp(x, nw, wgu, wd, EPS, kind="dot"),
        }[case]
    elif case in ("add_rms", "rms"):
        x = torch.randn(8192, H, device=dev, dtype=torch.float16, generator=g)
        r = torch.randn(8192, H, device=dev, dtype=torch.float16, generator=g)
        w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half()
        out = torch.empty_like(x)
        fn = ((lambda: fd.add_rms_norm(x, r, w, 1e-5, out=out, residual_out=r)) if case == "add_rms"
              else (lambda: fd.rms_norm(x, w, 1e-5, out=out)))
    elif case == "swiglu":
        a = torch.randn(2048, I, device=dev, dtype=torch.float16, generator=g)
        b = torch.randn(2048, I, device=dev, dtype=torch.float16, generator=g)
        out = torch.empty_like(a)
        fn = lambda: fd.swiglu(a, b, out=out)  # noqa: E731
    elif case == "rope":
        x = torch.randn(1, 2048, 32, 128, device=dev, dtype=torch.float16, generator=g)
        cos, sin = rope_tables(torch, 2048, 128, dev, torch.float16)
        out = torch.empty_like(x)
        fn = lambda: fd.rope(x, cos, sin, out=out)  # noqa: E731
    else:
        a = torch.empty(1 << 28, device=dev, dtype=bf).normal_()
        b = torch.empty_like(a)
        fn = lambda: K.launch_copy(b, a)  # noqa: E731
    for _ in range(5):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"ncu_case": case, "m": m, "launches": 5}))


def rope_tables(torch, positions, dim, device, dtype, theta=500000.0):
    """cos/sin [positions, 1, dim] for rotate-half RoPE: inv_freq[j] = theta^(-2j/dim)."""
    inv = theta ** (-torch.arange(0, dim, 2, dtype=torch.float32, device=device) / dim)
    f = torch.outer(torch.arange(positions, dtype=torch.float32, device=device), inv)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(dtype).view(positions, 1, dim), emb.sin().to(dtype).view(positions, 1, dim)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ops", action="store_true", help="skip the standalone-op measurements")
    ap.add_argument("--tp-collective", choices=("nvlink", "nccl"), default="nvlink",
                    help="N>1: partial sums over the NVLink exchange buffers (default) or NCCL all_reduce")
    ap.add_argument("--ncu-case", choices=NCU_CASES, default=None,
                    help="run a small fixed workload of one kernel for an ncu capture and exit")
    args = ap.parse_args()
    if args.ncu_case:
        run_ncu_case(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
