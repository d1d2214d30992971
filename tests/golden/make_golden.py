"""Generate the golden vectors in this folder from the reference itself.

Runs the reference package's own correctness formulation
(``fused_decode.reference`` -- PyTorch on CPU) on seeded inputs and stores the
inputs and outputs as ``golden.npz`` plus a ``manifest.json``.  The shapes
follow the reference's tests (tests/test_ops.py:42-171) and the benchmark
configurations, scaled down so the fixtures stay small.

This script needs the reference's ``src`` directory (the folder holding the
``fused_decode`` package), named by ``FUSED_DECODE_REF``, and is run by hand
in the build container:

    FUSED_DECODE_REF=<reference checkout>/src python tests/golden/make_golden.py

The GPU box never runs it; the committed fixtures travel instead.
"""

from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("FUSED_DECODE_REF")
if not REF:
    raise SystemExit("set FUSED_DECODE_REF to the reference's src directory")
sys.path.insert(0, REF)

from fused_decode import reference as R  # noqa: E402  (the reference's own oracle)

DT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def _np(t: torch.Tensor) -> tuple[np.ndarray, str]:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16), "bfloat16"
    if t.dtype == torch.float16:
        return t.numpy(), "float16"
    return t.float().numpy(), "float32"


def theta_tables(positions: int, dim: int, theta: float, dtype: torch.dtype):
    """Rotate-half cos/sin tables: inv_freq[j] = theta^(-2j/dim), emb = cat(f, f)."""
    inv = theta ** (-torch.arange(0, dim, 2, dtype=torch.float32) / dim)
    f = torch.outer(torch.arange(positions, dtype=torch.float32), inv)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


class Writer:
    def __init__(self) -> None:
        self.arrays: dict[str, np.ndarray] = {}
        self.cases: list[dict] = []

    def add(self, op: str, dtype: str, params: dict, inputs: dict, outputs: dict) -> None:
        cid = f"c{len(self.cases):03d}"
        entry = {"id": cid, "op": op, "dtype": dtype, "params": params, "inputs": {}, "outputs": {}}
        for kind, tensors in (("inputs", inputs), ("outputs", outputs)):
            for name, t in tensors.items():
                if t is None:
                    continue
                arr, dt = _np(t)
                key = f"{cid}/{name}"
                self.arrays[key] = arr
                entry[kind][name] = {"dtype": dt, "shape": list(t.shape)}
        self.cases.append(entry)

    def save(self) -> None:
        np.savez_compressed(os.path.join(HERE, "golden.npz"), **self.arrays)
        with open(os.path.join(HERE, "manifest.json"), "w") as f:
            json.dump({"generator": "tests/golden/make_golden.py",
                       "reference": "fused_decode.reference (src/fused_decode/reference.py)",
                       "torch": torch.__version__, "cases": self.cases}, f, indent=1)


def main() -> None:
    w = Writer()
    for dname in ("float16", "bfloat16"):
        dt = DT[dname]
        # rms_norm: reference tests/test_ops.py:42-48 shapes
        for shape in [(4, 128), (1, 4096), (3, 3072), (5, 100), (2, 8, 64)]:
            torch.manual_seed(0)
            x = torch.randn(*shape, dtype=dt)
            wt = torch.randn(shape[-1], dtype=dt)
            w.add("rms_norm", dname, {"eps": 1e-6}, {"x": x, "weight": wt},
                  {"y": R.rms_norm_reference(x, wt)})
        # fp32 weight (tests/test_ops.py:51-63)
        torch.manual_seed(1)
        x = torch.randn(48, 32, dtype=dt)
        wt = torch.randn(32, dtype=torch.float32)
        w.add("rms_norm", dname, {"eps": 1e-6, "layout": "transposed"}, {"x": x, "weight": wt},
              {"y": R.rms_norm_reference(x, wt)})
        # add+RMSNorm benchmark widths, 8 rows: w = 1 + 0.1 N(0,1), eps = 1e-5
        torch.manual_seed(0)
        x = torch.randn(8, 4096, dtype=dt)
        r = torch.randn(8, 4096, dtype=dt)
        wt = (1 + 0.1 * torch.randn(4096)).to(dt)
        w.add("rms_norm", dname, {"eps": 1e-5}, {"x": x, "weight": wt},
              {"y": R.rms_norm_reference(x, wt, 1e-5)})
        y, ro = R.add_rms_norm_reference(x, r, wt, 1e-5)
        w.add("add_rms_norm", dname, {"eps": 1e-5}, {"x": x, "residual": r, "weight": wt},
              {"y": y, "residual_out": ro})
        # add_rms_norm (tests/test_ops.py:66-81)
        torch.manual_seed(2)
        x = torch.randn(6, 256, dtype=dt)
        r = torch.randn(6, 256, dtype=dt)
        wt = torch.randn(256, dtype=dt)
        y, ro = R.add_rms_norm_reference(x, r, wt)
        w.add("add_rms_norm", dname, {"eps": 1e-6}, {"x": x, "residual": r, "weight": wt},
              {"y": y, "residual_out": ro})
        # swiglu (tests/test_ops.py:106-113) and the benchmark width
        for seed, shape, scale in [(5, (3, 128), 1.0), (0, (2, 14336), 1.0), (11, (4, 512), 30.0)]:
            torch.manual_seed(seed)
            g = (torch.randn(*shape) * scale).to(dt)
            u = torch.randn(*shape, dtype=dt)
            w.add("swiglu", dname, {}, {"gate": g, "up": u}, {"y": R.swiglu_reference(g, u)})
        # rope (tests/test_ops.py:91-103)
        torch.manual_seed(4)
        x = torch.randn(2, 8, 4, 128, dtype=dt)
        c = torch.randn(8, 1, 128, dtype=dt)
        s = torch.randn(8, 1, 128, dtype=dt)
        w.add("rope", dname, {}, {"x": x, "cos": c, "sin": s}, {"y": R.rope_reference(x, c, s)})
        x = torch.randn(2, 4, 8, 64, dtype=dt).transpose(1, 2).contiguous()
        c = torch.randn(1, 8, 1, 64, dtype=torch.float32)
        s = torch.randn(1, 8, 1, 64, dtype=torch.float32)
        w.add("rope", dname, {"layout": "transposed"}, {"x": x, "cos": c, "sin": s},
              {"y": R.rope_reference(x, c, s)})
        # rope with theta = 500000 tables (the RoPE benchmark tables), 16 positions
        torch.manual_seed(0)
        x = torch.randn(1, 16, 32, 128, dtype=dt)
        c, s = theta_tables(16, 128, 500000.0, dt)
        c, s = c.view(16, 1, 128), s.view(16, 1, 128)
        w.add("rope", dname, {"theta": 500000.0}, {"x": x, "cos": c, "sin": s},
              {"y": R.rope_reference(x, c, s)})
        # linear (tests/test_ops.py:116-142)
        for m, n, k in [(1, 64, 100), (3, 128, 128), (8, 256, 64)]:
            torch.manual_seed(6)
            x = (torch.randn(m, k) * k ** -0.5).to(dt)
            wt = (torch.randn(n, k) * k ** -0.5).to(dt)
            b = torch.randn(n, dtype=dt)
            w.add("linear", dname, {}, {"x": x, "weight": wt, "bias": b},
                  {"y": R.linear_reference(x, wt, b)})
        torch.manual_seed(7)
        x = (torch.randn(4, 128) * 128 ** -0.5).to(dt)
        wt = torch.randn(128, 64, dtype=dt).t().contiguous()  # [64, 128]
        row = torch.randn(4, 64, dtype=dt)
        w.add("linear", dname, {"layout": "transposed_weight"}, {"x": x, "weight": wt, "row_add": row},
              {"y": R.linear_reference(x, wt, row_add=row)})
        # GEMV sweep distributions: W ~ N(0, 0.02), x ~ N(0, 1), fp32 bias / row_add
        for m in (1, 2, 4, 8, 16):
            torch.manual_seed(100 + m)
            x = torch.randn(m, 2048, dtype=dt)
            wt = (torch.randn(40, 2048) * 0.02).to(dt)
            b = (torch.randn(40) * 0.02).float()
            row = torch.randn(m, 40, dtype=torch.float32)
            w.add("linear", dname, {}, {"x": x, "weight": wt, "bias": b, "row_add": row},
                  {"y": R.linear_reference(x, wt, b, row_add=row)})
        # post_attn_mlp (tests/test_ops.py:159-171) and Llama-3-8B MLP benchmark distributions
        torch.manual_seed(9)
        hid, inner = 64, 128
        x = torch.randn(4, hid, dtype=dt)
        nw = torch.randn(hid, dtype=dt)
        wgu = (torch.randn(inner * 2, hid) * hid ** -0.5).to(dt)
        wd = (torch.randn(hid, inner) * inner ** -0.5).to(dt)
        w.add("post_attn_mlp", dname, {"eps": 1e-6},
              {"hidden": x, "norm_weight": nw, "w_gate_up": wgu, "w_down": wd},
              {"y": R.post_attn_mlp_reference(x, nw, wgu, wd)})
        for m, hid, inner in ((1, 192, 320), (8, 128, 200)):
            torch.manual_seed(200 + m)
            x = torch.randn(m, hid, dtype=dt)
            nw = (1 + 0.1 * torch.randn(hid)).to(dt)
            wgu = (torch.randn(inner * 2, hid) * 0.02).to(dt)
            wd = (torch.randn(hid, inner) * 0.02).to(dt)
            w.add("post_attn_mlp", dname, {"eps": 1e-5},
                  {"hidden": x, "norm_weight": nw, "w_gate_up": wgu, "w_down": wd},
                  {"y": R.post_attn_mlp_reference(x, nw, wgu, wd, 1e-5)})
    # two-pass RMSNorm width (tests/test_ops.py:84-88)
    torch.manual_seed(3)
    x = torch.randn(2, 9000, dtype=torch.float16)
    wt = torch.randn(9000, dtype=torch.float16)
    w.add("rms_norm", "float16", {"eps": 1e-6}, {"x": x, "weight": wt}, {"y": R.rms_norm_reference(x, wt)})
    w.save()
    print(f"wrote {len(w.cases)} cases")


if __name__ == "__main__":
    main()
