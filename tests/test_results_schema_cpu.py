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
