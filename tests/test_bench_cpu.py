"""bench.py's contract on CPU: the reference arm's JSON line and the byte
counts the roofline divides by (the algorithmic bytes of the Llama-3-8B MLP
layer: weights once, hidden in, out, norm weight)."""

import io
import json
from contextlib import redirect_stdout
from types import SimpleNamespace

import bench


def test_layer_bytes():
    assert bench.layer_bytes(1) == 352_346_112
    assert bench.layer_bytes(8) == 352_460_800
    assert bench.gate_up_launch_bytes(1) == 2 * 14336 * 4096 * 2 + 4096 * 2 + 4096 * 2 + 14336 * 2
    assert bench.down_launch_bytes(1) == 4096 * 14336 * 2 + 14336 * 2 + 2 * 4096 * 2
    assert bench.layer_bytes(1, world=8) == (3 * 14336 * 4096 * 2) // 8 + 2 * 4096 * 2 + 4096 * 2


def test_reference_arm_line():
    args = SimpleNamespace(gpus=1, steps=1, warmup=3, m=1, tp_collective="nvlink")
    buf = io.StringIO()
    with redirect_stdout(buf):
        bench.run_reference(args)
    line = json.loads(buf.getvalue().strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "us/layer" and line["higher_is_better"] is False
    assert line["config"] == bench.workload_config(1, 1, "nvlink")
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["value"] > 0
