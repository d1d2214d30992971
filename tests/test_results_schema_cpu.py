"""The per-operator results module (``python -m fused_decode_b200.bench``):
host-side pieces on CPU -- the reference-schema row names and derived fields,
and the loud refusal without a GPU."""

import pytest
import torch

from fused_decode_b200 import bench as rb


def test_refuses_without_cuda(tmp_path):
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    with pytest.raises(SystemExit, match="CUDA is required"):
        rb.main(["--quick", "--out", str(tmp_path / "r.json")])


def test_row_fields_and_names():
    roof = {"copy_gbs": 6500.0, "l2_bytes": 126 * 2**20, "cublas_tflops": 1500.0}
    t = rb.Table(roof, compile_eager=False)
    bw = t.bandwidth(134_225_920, 25.0)
    assert bw["bytes"] == 134_225_920 and not bw["fits_l2"]
    assert bw["gbs"] == pytest.approx(134_225_920 / 25e-6 / 1e9)
    assert bw["pct_copy_roof"] == pytest.approx(bw["gbs"] / 6500.0 * 100.0)
    assert t.bandwidth(1024, 1.0)["fits_l2"]
    # the reference formats row names with the torch dtype's repr
    assert f"rms_norm 8192x4096 {torch.float16}" == "rms_norm 8192x4096 torch.float16"
    assert f"rope {tuple((1, 2048, 32, 128))} {torch.bfloat16}" == "rope (1, 2048, 32, 128) torch.bfloat16"
    row = t.add({"name": "x", "us": 2.0, "eager_us": 4.0})
    assert t.rows == [row]
    assert rb._speedup(4.0, 2.0) == 2.0 and rb._speedup(None, 2.0) is None


# ---- the row set against the reference's published table ------------------
import json  # noqa: E402
import os  # noqa: E402

_HERE = os.path.dirname(os.path.abspath(__file__))
_REF = json.load(open(os.path.join(_HERE, "golden", "reference_results_row_names.json"), encoding="utf-8"))
# Rows of the published file that the current reference bench no longer
# writes: its launcher rejects M > 16 (kernels.py:759-760), so only the
# "dispatch" rows remain at M = 32 and 128.
_STALE = {f"linear M={m} N=4096 K=4096 dot torch.{dt}" for m in (32, 128) for dt in ("float16", "bfloat16")}
_COMPILE_ONLY = {"compile_default_us", "compile_reduce-overhead_us", "speedup_vs_compile_default",
                 "speedup_vs_compile_reduce-overhead"}


def test_row_plan_is_the_reference_row_set():
    plan = rb.row_names(torch.float16) + rb.row_names(torch.bfloat16)
    assert plan == [n for n in _REF["names"] if n not in _STALE]
    assert len(plan) == 60 and len(set(plan)) == 60
    quick = rb.row_names(torch.float16, quick=True)
    assert set(quick) <= set(plan) | {"linear M=32 N=4096 K=4096 dispatch torch.float16"}


def test_committed_results_file_has_the_reference_schema():
    with open(os.path.join(_HERE, "..", "results", "b200.json"), encoding="utf-8") as f:
        doc = json.load(f)
    assert all(k in doc for k in _REF["top_level_keys"])
    assert [r["name"] for r in doc["rows"]] == rb.row_names(torch.float16) + rb.row_names(torch.bfloat16)
    keys = {k for r in doc["rows"] for k in r}
    assert set(_REF["row_keys"]) - _COMPILE_ONLY <= keys
    assert "B200" in doc["gpu"]["name"]
    for r in doc["rows"]:
        assert r["us"] > 0, r["name"]
        if "max_abs_vs_fp32" in r:
            # at most one bf16 ulp of these outputs (|y| < 8) against the fp32 references
            assert r["max_abs_vs_fp32"] <= 0.05, r["name"]
