"""Results table in the reference's schema, measured on this GPU.

    python -m fused_decode_b200.bench --out results/b200.json
    python -m fused_decode_b200.bench --compile --out results/b200.json
    python -m fused_decode_b200.bench --quick

Writes the same JSON document as the reference's ``python -m fused_decode.bench``
(src/fused_decode/bench.py:531-584): ``gpu``, ``torch``, ``triton``, the two
matmul precision flags, ``clocks_under_load``, one ``roofline`` entry per
dtype and one ``rows`` entry per measured case, with the reference's row names
(``"rms_norm 8192x4096 torch.float16"``, ``"linear M=1 N=4096 K=4096 dot
torch.bfloat16"``, ...) and fields (``us``, ``eager_us``, ``speedup_vs_eager``,
``gbs``, ``pct_copy_roof``, ``bytes``, ``max_abs*``, ``mv_us``,
``issued_tflops`` ...).  A results file from the reference and one from here
can therefore be joined row by row.

Timing follows the reference's method so the rows compare: CUDA-event median
of 5 rounds of back-to-back calls after warm-up, useful bytes over that time in
decimal GB.  Inputs are not rotated, so a row whose bytes fit the L2 cache
(126 MB on B200) can read from L2 on repeated calls; each row records
``fits_l2``.  Added fields: ``max_abs_vs_fp32`` on every checked row (against
``fused_decode_b200.reference``), ``l2_bytes`` and ``copy_elems`` in the
roofline entry, and ``cuda_graph_rotating_us`` on the MLP rows (weights
rotated across copies larger than L2, replayed in one graph).  The repository
root's ``bench.py`` holds the headline measurement (32-layer MLP stack);
this module is the per-operator table.
"""

from __future__ import annotations

import argparse
import json
import statistics
import subprocess
import threading
import time
from pathlib import Path

import torch
import torch.nn.functional as F

import fused_decode_b200 as fd
from fused_decode_b200 import kernels as K
from fused_decode_b200 import reference as R

LLAMA_H = 4096
LLAMA_I = 14336
COPY_ELEMS = 256 * 1024 * 1024  # 512 MB per fp16 buffer: the copy roof streams from HBM


# ------------------------------------------------------------------ timing
def time_us(fn, iters: int, warmup: int = 10, rounds: int = 5) -> float:
    """Median over ``rounds`` of the mean device time (us) of ``iters``
    back-to-back calls, CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per_call = []
    for _ in range(rounds):
        t0.record()
        for _ in range(iters):
            fn()
        t1.record()
        torch.cuda.synchronize()
        per_call.append(t0.elapsed_time(t1) * 1e3 / iters)
    return statistics.median(per_call)


def graph_us(calls, inner: int = 30, rounds: int = 5):
    """Per-call device time (us) of ``inner`` calls (rotating over ``calls``)
    captured in one CUDA graph; (None, error text) when capture fails."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # workspaces are per stream: create them before capture
        for c in calls:
            c()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(g, stream=side):
            for j in range(inner):
                calls[j % len(calls)]()
    except Exception as exc:  # reported in the row, as the reference does
        return None, f"{type(exc).__name__}: {exc}"
    us = time_us(g.replay, iters=1, warmup=3, rounds=rounds) / inner
    del g
    return us, None


def _speedup(base_us, ours_us):
    return base_us / ours_us if base_us and ours_us else None


def _max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.float() - b.float()).abs().max().item()


# ------------------------------------------------------------------ environment
def _smi(query: str, timeout: float) -> str:
    """One nvidia-smi query for the current CUDA device, selected by UUID
    (CUDA_VISIBLE_DEVICES may renumber devices), else by index."""
    dev = torch.cuda.current_device()
    ids = [str(dev)]
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    if uuid is not None:
        ids.insert(0, f"GPU-{uuid}")
    last: Exception = OSError("nvidia-smi")
    for gid in ids:
        try:
            return subprocess.check_output(
                ["nvidia-smi", f"--query-gpu={query}", "--format=csv,noheader,nounits", f"--id={gid}"],
                text=True, timeout=timeout, stderr=subprocess.DEVNULL).strip()
        except (subprocess.SubprocessError, OSError) as exc:
            last = exc
    raise last


def gpu_info() -> dict:
    fields = "name,driver_version,memory.total,clocks.max.sm,clocks.max.mem,power.max_limit"
    keys = ["name", "driver", "memory_mib", "max_sm_mhz", "max_mem_mhz", "max_power_w"]
    try:
        text = _smi(fields, timeout=10)
        info = dict(zip(keys, (p.strip() for p in text.splitlines()[0].split(","))))
    except (subprocess.SubprocessError, OSError, IndexError):
        info = {"name": torch.cuda.get_device_name()}
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    info["sm_count"] = props.multi_processor_count
    info["capability"] = f"sm_{props.major}{props.minor}"
    if "B200" in info.get("name", "") and "max_mem_mhz" in info:
        # HBM3e: 8 stacks x 1024-bit, double data rate on the reported clock
        info["theoretical_gbs"] = float(info["max_mem_mhz"]) * 1e6 * 2 * 8192 / 8 / 1e9
        info["theoretical_gbs_note"] = "mem_clock_mhz * 2 * 8192-bit / 8, from nvidia-smi max memory clock"
    return info


def clocks_under_load(seconds: float = 1.5) -> dict:
    """Median power, SM/memory clocks and utilisation sampled by nvidia-smi
    while an fp16 matmul loop keeps the GPU busy."""
    a = torch.randn(4096, 4096, device="cuda", dtype=torch.float16)
    b = torch.empty_like(a)
    samples: list[list[float]] = []
    stop = threading.Event()

    def poll() -> None:
        q = "power.draw,clocks.sm,clocks.mem,utilization.gpu"
        while not stop.is_set():
            try:
                samples.append([float(v) for v in _smi(q, timeout=2).split(",")])
            except (subprocess.SubprocessError, OSError, ValueError):
                pass
            stop.wait(0.2)

    th = threading.Thread(target=poll, daemon=True)
    th.start()
    end = time.perf_counter() + seconds
    while time.perf_counter() < end:
        torch.mm(a, a, out=b)
    torch.cuda.synchronize()
    stop.set()
    th.join(timeout=3)
    if not samples:
        return {}
    cols = list(zip(*samples))
    out = {k: statistics.median(c) for k, c in zip(("power_w", "sm_mhz", "mem_mhz", "util_pct"), cols)}
    out["samples"] = len(samples)
    return out


def roofline(dtype: torch.dtype) -> dict:
    """Measured copy and triad bandwidth (this library's kernels) and cuBLAS
    matmul throughput, the denominators of the rows' percentages."""
    n = COPY_ELEMS
    a = torch.randn(n, device="cuda", dtype=dtype)
    b = torch.randn(n, device="cuda", dtype=dtype)
    c = torch.empty(n, device="cuda", dtype=dtype)
    item = a.element_size()
    copy_us = time_us(lambda: K.launch_copy(c, a), iters=10, warmup=3)
    triad_us = time_us(lambda: K.launch_triad(a, b, c, 1.25), iters=10, warmup=3)
    del a, b, c
    side = 8192
    x = torch.randn(side, side, device="cuda", dtype=dtype)
    y = torch.randn(side, side, device="cuda", dtype=dtype)
    mm_us = time_us(lambda: torch.mm(x, y), iters=10, warmup=5, rounds=3)
    return {
        "dtype": str(dtype).replace("torch.", ""),
        "copy_gbs": 2 * n * item / copy_us / 1e3,
        "triad_gbs": 3 * n * item / triad_us / 1e3,
        "copy_us": copy_us,
        "triad_us": triad_us,
        "copy_elems": n,
        "cublas_tflops": 2.0 * side**3 / mm_us / 1e6,
        "cublas_mm_us": mm_us,
        "cublas_mm_n": side,
        "l2_bytes": torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size,
    }


# ------------------------------------------------------------------ rows
class Table:
    """Collects rows; shared fields (bandwidth, roof %, L2 fit) in one place."""

    def __init__(self, roof: dict, compile_eager: bool) -> None:
        self.roof = roof
        self.compile_eager = compile_eager
        self.rows: list[dict] = []

    def add(self, row: dict) -> dict:
        self.rows.append(row)
        extra = f"eager {row['eager_us']:.2f}" if row.get("eager_us") else ""
        print(f"{row['name']}: {row['us']:.2f} us {extra}", flush=True)
        return row

    def bandwidth(self, nbytes: int, us: float) -> dict:
        gbs = nbytes / us / 1e3
        return {"gbs": gbs, "pct_copy_roof": gbs / self.roof["copy_gbs"] * 100.0, "bytes": nbytes,
                "fits_l2": nbytes <= self.roof["l2_bytes"]}

    def pointwise(self, name, ours, eager, nbytes, checks=None, compile_this=False) -> dict:
        iters = 100 if nbytes < 1_000_000 else 30
        us = time_us(ours, iters)
        eager_us = time_us(eager, iters)
        row = {"name": name, "us": us, "eager_us": eager_us, "speedup_vs_eager": _speedup(eager_us, us)}
        row.update(self.bandwidth(nbytes, us))
        for key, fn in (checks or {}).items():
            row[key] = fn()
        if compile_this and self.compile_eager:
            _compile_into(row, eager, "default", us, iters=max(10, iters // 2))
        return self.add(row)


def _compile_into(row: dict, eager, mode: str, ours_us: float, iters: int) -> None:
    try:
        compiled = torch.compile(eager, mode=mode, dynamic=False)
        c_us = time_us(compiled, iters=iters, warmup=5, rounds=3)  # compilation stays in warm-up
        row[f"compile_{mode}_us"] = c_us
        row[f"speedup_vs_compile_{mode}"] = _speedup(c_us, ours_us)
    except Exception as exc:
        row[f"compile_{mode}_error"] = f"{type(exc).__name__}: {exc}"


# ------------------------------------------------------------------ the row plan
# Shapes and row names of the table (the reference's, src/fused_decode/
# bench.py:193-448).  The timing code below and row_names() both read these,
# so the row set can be checked without a GPU.
def norm_shapes(quick: bool) -> list[tuple[int, int]]:
    return [(2048, LLAMA_H), (1, LLAMA_H)] if quick else [(8192, LLAMA_H), (2048, LLAMA_H), (1, LLAMA_H)]


def swiglu_rows(quick: bool) -> tuple[int, ...]:
    return (2048,) if quick else (1, 2048)


def rope_cases(quick: bool) -> list[tuple[tuple[int, ...], tuple[int, ...]]]:
    """(x shape, cos/sin shape): cos/sin broadcast over heads as [S, 1, D]."""
    return [((1, 2048, 32, 128), (2048, 1, 128))] + ([] if quick else [((1, 1, 32, 128), (1, 1, 128))])


def linear_shapes(quick: bool) -> list[tuple[int, int, int]]:
    h, i = LLAMA_H, LLAMA_I
    if quick:
        return [(1, h, h), (8, h, h), (32, h, h)]
    return [(1, h, h), (1, h, i), (1, i, h), (4, h, h), (8, h, h), (16, h, h), (32, h, h), (128, h, h)]


def linear_kinds(m: int) -> tuple[str, ...]:
    """Kinds timed per shape: both GEMV kinds up to the GEMV's batch limit."""
    return ("dot", "simt") if m <= fd.DECODE_LINEAR_MAX_M else ()


def mlp_cases(quick: bool) -> list[tuple[int, tuple]]:
    """(batch rows, kinds); kind None is the default dispatcher."""
    return [(1, (None, "simt"))] + ([] if quick else [(8, (None,))])


def name_norm(op: str, rows_n: int, h: int, dtype) -> str:
    return f"{op} {rows_n}x{h} {dtype}"


def name_swiglu(rows_n: int, dtype) -> str:
    return f"swiglu {rows_n}x{LLAMA_I} {dtype}"


def name_rope(xs, dtype) -> str:
    return f"rope {tuple(xs)} {dtype}"


def name_linear(m: int, n: int, k: int, kind: str, dtype) -> str:
    return f"linear M={m} N={n} K={k} {kind} {dtype}"


def name_mlp(m: int, kind, dtype) -> str:
    return f"post_attn_mlp M={m} {'default' if kind is None else kind} {dtype}"


def row_names(dtype, quick: bool = False) -> list[str]:
    """The rows one dtype contributes, in the order the table writes them."""
    names = []
    for rows_n, h in norm_shapes(quick):
        names += [name_norm("rms_norm", rows_n, h, dtype), name_norm("add_rms_norm", rows_n, h, dtype)]
    names += [name_swiglu(rows_n, dtype) for rows_n in swiglu_rows(quick)]
    names += [name_rope(xs, dtype) for xs, _ in rope_cases(quick)]
    for m, n, k in linear_shapes(quick):
        if m > 1:
            names.append(name_linear(m, n, k, "dispatch", dtype))
        names += [name_linear(m, n, k, kind, dtype) for kind in linear_kinds(m)]
    for m, kinds in mlp_cases(quick):
        names += [name_mlp(m, kind, dtype) for kind in kinds]
    return names


def bench_rows_ops(t: Table, dtype: torch.dtype, quick: bool) -> None:
    """RMSNorm, add+RMSNorm, SwiGLU and RoPE at the reference's bench shapes
    (src/fused_decode/bench.py:193-300)."""
    item = torch.empty((), dtype=dtype).element_size()
    for rows_n, h in norm_shapes(quick):
        x = torch.randn(rows_n, h, device="cuda", dtype=dtype)
        res = torch.randn_like(x)
        w = torch.randn(h, device="cuda", dtype=dtype)
        t.pointwise(
            name_norm("rms_norm", rows_n, h, dtype),
            lambda: fd.rms_norm(x, w), lambda: F.rms_norm(x, (h,), w, 1e-6),
            (2 * rows_n * h + h) * item,
            checks={"max_abs": lambda: _max_abs(fd.rms_norm(x, w), F.rms_norm(x, (h,), w, 1e-6)),
                    "max_abs_vs_fp32": lambda: _max_abs(fd.rms_norm(x, w), R.rms_norm_reference(x, w))},
        )
        t.pointwise(
            name_norm("add_rms_norm", rows_n, h, dtype),
            lambda: fd.add_rms_norm(x, res, w), lambda: F.rms_norm(x + res, (h,), w, 1e-6),
            (4 * rows_n * h + h) * item,
            checks={"max_abs_vs_fp32": lambda: max(
                _max_abs(a, b) for a, b in zip(fd.add_rms_norm(x, res, w), R.add_rms_norm_reference(x, res, w)))},
            compile_this=dtype == torch.float16 and rows_n == 2048,
        )
    for rows_n in swiglu_rows(quick):
        g = torch.randn(rows_n, LLAMA_I, device="cuda", dtype=dtype)
        u = torch.randn_like(g)
        t.pointwise(
            name_swiglu(rows_n, dtype),
            lambda: fd.swiglu(g, u), lambda: F.silu(g) * u, 3 * g.numel() * item,
            checks={"max_abs_vs_fp32": lambda: _max_abs(fd.swiglu(g, u), R.swiglu_reference(g, u))},
            compile_this=dtype == torch.float16 and rows_n == 2048,
        )
    for xs, cs in rope_cases(quick):
        x = torch.randn(*xs, device="cuda", dtype=dtype)
        cos = torch.randn(*cs, device="cuda", dtype=dtype)
        sin = torch.randn(*cs, device="cuda", dtype=dtype)

        def eager(x=x, cos=cos, sin=sin):
            x1, x2 = x.chunk(2, dim=-1)
            c, s = cos.expand_as(x), sin.expand_as(x)
            c1, c2 = c.chunk(2, dim=-1)
            s1, s2 = s.chunk(2, dim=-1)
            return torch.cat((x1 * c1 - x2 * s1, x2 * c2 + x1 * s2), dim=-1)

        t.pointwise(
            name_rope(xs, dtype),
            lambda: fd.rope(x, cos, sin), eager, 2 * x.nbytes + cos.nbytes + sin.nbytes,
            checks={"max_abs": lambda: _max_abs(fd.rope(x, cos, sin), R.rope_reference(x, cos, sin))},
            compile_this=dtype == torch.float16 and xs[1] == 2048,
        )


def bench_rows_linear(t: Table, dtype: torch.dtype, quick: bool) -> None:
    """``linear_decode`` per kind, the default dispatcher above M=1, cuBLAS
    (``F.linear``) and ``torch.mv`` beside it (src/fused_decode/bench.py:303-385).

    Issued flops count the batch columns the tensor-core path computes: the
    ``dot`` consumers run m16n8k16 with the batch as the 8-wide operand, so
    M<=8 issues 8 columns and M<=16 issues 16; ``simt`` issues M."""
    item = torch.empty((), dtype=dtype).element_size()
    for m, n, k in linear_shapes(quick):
        x = torch.randn(m, k, device="cuda", dtype=dtype) * k**-0.5
        w = torch.randn(n, k, device="cuda", dtype=dtype) * k**-0.5
        nbytes = (m * k + n * k + m * n) * item
        eager_us = time_us(lambda: F.linear(x, w), iters=50 if m <= 16 else 20)
        mv_us = time_us(lambda: torch.mv(w, x.reshape(-1)), iters=50) if m == 1 else None
        if m > 1:
            us = time_us(lambda: fd.linear_decode(x, w), iters=30, warmup=5, rounds=3)
            t.add({
                "name": name_linear(m, n, k, "dispatch", dtype), "us": us, "eager_us": eager_us,
                "mv_us": mv_us, "speedup_vs_eager": _speedup(eager_us, us), "bytes": nbytes,
                "note": (f"default dispatcher: hand-written GEMV up to M={fd.DECODE_LINEAR_MAX_M}, "
                         "cuBLAS above"),
            })
        if not linear_kinds(m):
            continue
        ref = R.linear_reference(x, w)
        cublas = F.linear(x, w)
        for kind in linear_kinds(m):
            us = time_us(lambda: fd.linear_decode(x, w, kind=kind), iters=50)
            ours = fd.linear_decode(x, w, kind=kind)
            cols = (8 if m <= 8 else 16) if kind == "dot" else m
            issued = 2.0 * cols * n * k / us / 1e6
            row = {"name": name_linear(m, n, k, kind, dtype), "us": us, "eager_us": eager_us,
                   "mv_us": mv_us, "speedup_vs_eager": _speedup(eager_us, us),
                   "speedup_vs_mv": _speedup(mv_us, us)}
            row.update(t.bandwidth(nbytes, us))
            row.update({
                "useful_tflops": 2.0 * m * n * k / us / 1e6,
                "issued_tflops": issued,
                "issued_pct_cublas_peak": issued / t.roof["cublas_tflops"] * 100.0,
                "max_abs_vs_fp32": _max_abs(ours, ref),
                "max_abs_vs_cublas": _max_abs(ours, cublas),
            })
            t.add(row)


def _mlp_weights(dtype, m, copies=1):
    g = torch.Generator(device="cuda").manual_seed(1234 + m)
    hidden = torch.randn(m, LLAMA_H, device="cuda", dtype=dtype, generator=g)
    norm_w = torch.ones(LLAMA_H, device="cuda", dtype=dtype)
    sets = []
    for _ in range(copies):
        w_gu = torch.randn(2 * LLAMA_I, LLAMA_H, device="cuda", dtype=dtype, generator=g) * LLAMA_H**-0.5
        w_dn = torch.randn(LLAMA_H, LLAMA_I, device="cuda", dtype=dtype, generator=g) * LLAMA_I**-0.5
        sets.append((w_gu, w_dn))
    return hidden, norm_w, sets


def bench_rows_mlp(t: Table, dtype: torch.dtype, quick: bool) -> None:
    """``post_attn_mlp`` at Llama-3-8B widths against its eager PyTorch
    formulation (src/fused_decode/bench.py:388-448), plus two graph times:
    the reference's (one weight set, L2-warm) and one with the weights rotated
    across copies that together exceed L2, which is what a layer stack sees."""
    for m, kinds in mlp_cases(quick):
        hidden, norm_w, sets = _mlp_weights(dtype, m, copies=2)
        w_gu, w_dn = sets[0]

        def eager(w_gu=w_gu, w_dn=w_dn):
            hh = F.rms_norm(hidden, (LLAMA_H,), norm_w, 1e-6)
            gate, up = F.linear(hh, w_gu).split(LLAMA_I, dim=-1)
            return F.linear(F.silu(gate) * up, w_dn) + hidden

        for kind in kinds:
            def ours(w_gu=w_gu, w_dn=w_dn, kind=kind):
                return fd.post_attn_mlp(hidden, norm_w, w_gu, w_dn, kind=kind)

            us = time_us(ours, iters=30, warmup=10)
            eager_us = time_us(eager, iters=30, warmup=10)
            with torch.no_grad():
                got = ours()
                row = {"name": name_mlp(m, kind, dtype),
                       "us": us, "eager_us": eager_us, "speedup_vs_eager": _speedup(eager_us, us),
                       "max_abs_vs_eager": _max_abs(got, eager()),
                       "max_abs_vs_fp32": _max_abs(got, R.post_attn_mlp_reference(hidden, norm_w, w_gu, w_dn))}
            nbytes = (3 * LLAMA_I * LLAMA_H + 2 * m * LLAMA_H + LLAMA_H) * hidden.element_size()
            row.update(t.bandwidth(nbytes, us))
            if kind is None and dtype == torch.float16 and t.compile_eager:
                for mode in ("default", "reduce-overhead"):
                    _compile_into(row, eager, mode, us, iters=30)
            row["cuda_graph_us"], err = graph_us([ours])
            if err:
                row["cuda_graph_error"] = err
            rot, _ = graph_us([lambda s=s, kind=kind: fd.post_attn_mlp(hidden, norm_w, s[0], s[1], kind=kind)
                               for s in sets])
            row["cuda_graph_rotating_us"] = rot
            t.add(row)
        del sets


# ------------------------------------------------------------------ main
def _print_table(rows: list[dict]) -> None:
    print("\nname | us | eager_us | speedup | gbs | pct_roof")
    for r in rows:
        f = lambda key, spec: format(r[key], spec) if r.get(key) is not None else ""  # noqa: E731
        sp = f"{r['speedup_vs_eager']:.2f}x" if r.get("speedup_vs_eager") else ""
        print(f"{r['name']} | {r['us']:.2f} | {f('eager_us', '.2f')} | {sp} | {f('gbs', '.1f')} | "
              f"{f('pct_copy_roof', '.1f')}")


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Per-operator results table (reference schema) on this GPU")
    p.add_argument("--out", type=Path, default=Path("results/latest.json"))
    p.add_argument("--compile", action="store_true", help="also time torch.compile of the eager formulations")
    p.add_argument("--quick", action="store_true", help="fp16 headline shapes only")
    p.add_argument("--dtype", choices=("float16", "bfloat16", "both"), default="both")
    args = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("CUDA is required")
    torch.manual_seed(0)
    torch.cuda.manual_seed(0)
    if args.quick or args.dtype == "float16":
        dtypes = [torch.float16]
    elif args.dtype == "bfloat16":
        dtypes = [torch.bfloat16]
    else:
        dtypes = [torch.float16, torch.bfloat16]
    doc = {
        "gpu": gpu_info(),
        "torch": torch.__version__,
        "triton": None,
        "backend": f"fused_decode_b200 {fd.__version__}: hand-written CUDA for sm_100a (libfd_b200.so)",
        "cuda": torch.version.cuda,
        "allow_tf32": bool(torch.backends.cuda.matmul.allow_tf32),
        "allow_fp16_reduced_precision_reduction": bool(
            torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction),
        "clocks_under_load": clocks_under_load(),
        "timing": ("CUDA-event median of 5 rounds of back-to-back calls after warm-up; inputs not rotated "
                   "(rows with fits_l2 may read from L2)"),
        "roofline": [],
        "rows": [],
    }
    print(json.dumps({k: doc[k] for k in ("gpu", "torch", "cuda", "clocks_under_load")}, indent=2))
    args.out.parent.mkdir(parents=True, exist_ok=True)
    for dtype in dtypes:
        roof = roofline(dtype)
        doc["roofline"].append(roof)
        print(f"roof {dtype}: copy {roof['copy_gbs']:.1f} GB/s, triad {roof['triad_gbs']:.1f} GB/s, "
              f"cublas {roof['cublas_tflops']:.1f} TFLOP/s", flush=True)
        t = Table(roof, args.compile)
        bench_rows_ops(t, dtype, args.quick)
        bench_rows_linear(t, dtype, args.quick)
        bench_rows_mlp(t, dtype, args.quick)
        doc["rows"].extend(t.rows)
        args.out.write_text(json.dumps(doc, indent=2) + "\n", encoding="utf-8")
        torch.cuda.empty_cache()
    _print_table(doc["rows"])
    print(f"wrote {args.out}")


if __name__ == "__main__":
    main()
