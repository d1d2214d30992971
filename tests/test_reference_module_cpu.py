"""``fused_decode_b200.reference`` (the torch fp32 references callers' tests
compare against) reproduces the reference package's golden outputs exactly:
the golden vectors were made by the reference's own ``fused_decode.reference``
on the CPU, so the same formulation must give the same bits."""

import pytest
import torch

from fused_decode_b200 import reference as R
from tests._golden import load_golden, to_torch

CASES = load_golden()


def _run(case):
    t = {k: to_torch(v, device="cpu") for k, v in case["inputs"].items()}
    eps = case["params"].get("eps", 1e-6)
    op = case["op"]
    if op == "rms_norm":
        return {"y": R.rms_norm_reference(t["x"], t["weight"], eps)}
    if op == "add_rms_norm":
        y, ro = R.add_rms_norm_reference(t["x"], t["residual"], t["weight"], eps)
        return {"y": y, "residual_out": ro}
    if op == "swiglu":
        return {"y": R.swiglu_reference(t["gate"], t["up"])}
    if op == "rope":
        return {"y": R.rope_reference(t["x"], t["cos"], t["sin"])}
    if op == "linear":
        return {"y": R.linear_reference(t["x"], t["weight"], t.get("bias"), t.get("row_add"))}
    if op == "post_attn_mlp":
        return {"y": R.post_attn_mlp_reference(t["hidden"], t["norm_weight"], t["w_gate_up"],
                                               t["w_down"], eps)}
    raise AssertionError(op)


@pytest.mark.parametrize("case", CASES, ids=[c["id"] + "-" + c["op"] for c in CASES])
def test_reference_module_matches_golden(case):
    got = _run(case)
    assert set(got) == set(case["outputs"])
    for name, want in case["outputs"].items():
        w = to_torch(want, device="cpu")
        assert got[name].dtype == w.dtype and got[name].shape == w.shape, name
        assert torch.equal(got[name], w), (case["id"], name, (got[name].float() - w.float()).abs().max().item())


def test_reference_module_names():
    for name in ("rms_norm_reference", "add_rms_norm_reference", "swiglu_reference",
                 "rope_reference", "linear_reference", "post_attn_mlp_reference"):
        assert callable(getattr(R, name))
