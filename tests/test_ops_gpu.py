"""Parity of the CUDA operators with the reference's formulation.

The first half ports the reference's own test file (tests/test_ops.py:1-187)
with the import switched to fused_decode_b200 and the comparator switched to
the CPU oracle (a numpy restatement of reference.py, pinned to the reference
by tests/test_oracle_golden.py).  The tolerance table is the reference's
(tests/test_ops.py:27-35).  The second half runs every golden vector through
the CUDA path and compares with the reference's stored outputs.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import fd_oracle as O
from tests._golden import load_golden, to_torch

pytestmark = pytest.mark.gpu

DTYPES = [torch.float16, torch.bfloat16]
_NAME = {torch.float16: "float16", torch.bfloat16: "bfloat16"}


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.fail("CUDA GPU required for -m gpu tests")
    import fused_decode_b200._capi as capi

    capi.load()  # fail loudly if the native library is missing


def _np(t):
    return t.detach().float().cpu().numpy()


def _tol(dtype, kind):
    # reference tests/test_ops.py:27-35
    if kind == "linear":
        if dtype == torch.float16:
            return {"rtol": 2e-2, "atol": 2e-2}
        return {"rtol": 4e-2, "atol": 4e-2}
    if dtype == torch.float16:
        return {"rtol": 1e-2, "atol": 5e-3}
    return {"rtol": 2e-2, "atol": 2e-2}


def _assert(actual, expected_np, dtype, kind="pointwise"):
    expected = torch.from_numpy(np.ascontiguousarray(expected_np)).to(actual.device, torch.float32)
    assert actual.shape == expected.shape
    torch.testing.assert_close(actual.float(), expected, **_tol(dtype, kind))


from fused_decode_b200 import (  # noqa: E402
    add_rms_norm,
    linear_decode,
    post_attn_mlp,
    rms_norm,
    rope,
    swiglu,
)


# ------------------------------------------------------------------ reference test port
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(4, 128), (1, 4096), (3, 3072), (5, 100), (2, 8, 64)])
def test_rms_norm(dtype, shape):
    torch.manual_seed(0)
    x = torch.randn(*shape, device="cuda", dtype=dtype)
    w = torch.randn(shape[-1], device="cuda", dtype=dtype)
    _assert(rms_norm(x, w), O.rms_norm(_np(x), _np(w), 1e-6, _NAME[dtype]), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_rms_norm_strided_and_fp32_weight(dtype):
    torch.manual_seed(1)
    base = torch.randn(32, 48, device="cuda", dtype=dtype)
    x = base.t()
    assert x.stride(-1) != 1
    w = torch.randn(x.shape[-1], device="cuda", dtype=torch.float32)
    _assert(rms_norm(x, w), O.rms_norm(_np(x), _np(w), 1e-6, _NAME[dtype]), dtype)

    y = torch.randn(7, 9, 32, device="cuda", dtype=dtype).transpose(0, 1)
    assert not y.is_contiguous()
    wy = torch.ones(y.shape[-1], device="cuda", dtype=dtype)
    _assert(rms_norm(y, wy), O.rms_norm(_np(y), _np(wy), 1e-6, _NAME[dtype]), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_add_rms_norm_inplace(dtype):
    torch.manual_seed(2)
    x = torch.randn(6, 256, device="cuda", dtype=dtype)
    residual = torch.randn(6, 256, device="cuda", dtype=dtype)
    w = torch.randn(256, device="cuda", dtype=dtype)
    y_ref, r_ref = O.add_rms_norm(_np(x), _np(residual), _np(w), 1e-6, _NAME[dtype])
    y, residual_out = add_rms_norm(x, residual, w)
    _assert(y, y_ref, dtype)
    _assert(residual_out, r_ref, dtype)

    residual2 = residual.clone()
    y2, residual_back = add_rms_norm(x, residual2, w, residual_out=residual2)
    assert residual_back.data_ptr() == residual2.data_ptr()
    _assert(y2, y_ref, dtype)
    _assert(residual2, r_ref, dtype)


def test_rms_two_pass():
    torch.manual_seed(3)
    x = torch.randn(2, 9000, device="cuda", dtype=torch.float16)
    w = torch.randn(9000, device="cuda", dtype=torch.float16)
    _assert(rms_norm(x, w), O.rms_norm(_np(x), _np(w), 1e-6, "float16"), torch.float16)


@pytest.mark.parametrize("dtype", DTYPES)
def test_rope_broadcast_and_transpose(dtype):
    torch.manual_seed(4)
    x = torch.randn(2, 8, 4, 128, device="cuda", dtype=dtype)
    cos = torch.randn(8, 1, 128, device="cuda", dtype=dtype)
    sin = torch.randn(8, 1, 128, device="cuda", dtype=dtype)
    _assert(rope(x, cos, sin), O.rope(_np(x), _np(cos), _np(sin), _NAME[dtype]), dtype)

    transposed = torch.randn(2, 4, 8, 64, device="cuda", dtype=dtype).transpose(1, 2)
    assert not transposed.is_contiguous()
    cos_t = torch.randn(1, 8, 1, 64, device="cuda", dtype=torch.float32)
    sin_t = torch.randn(1, 8, 1, 64, device="cuda", dtype=torch.float32)
    _assert(rope(transposed, cos_t, sin_t), O.rope(_np(transposed), _np(cos_t), _np(sin_t), _NAME[dtype]), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_swiglu_strided_halves(dtype):
    torch.manual_seed(5)
    rows, inner = 3, 128
    packed = torch.randn(rows, inner * 2, device="cuda", dtype=dtype)
    gate, up = packed.split(inner, dim=-1)
    assert not gate.is_contiguous()
    _assert(swiglu(gate, up), O.swiglu(_np(gate), _np(up), _NAME[dtype]), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("kind", ["dot", "simt"])
@pytest.mark.parametrize("m,n,k", [(1, 64, 100), (3, 128, 128), (8, 256, 64)])
def test_linear_small(dtype, kind, m, n, k):
    torch.manual_seed(6)
    x = torch.randn(m, k, device="cuda", dtype=dtype) * (k**-0.5)
    w = torch.randn(n, k, device="cuda", dtype=dtype) * (k**-0.5)
    bias = torch.randn(n, device="cuda", dtype=dtype)
    y = linear_decode(x, w, bias, kind=kind)
    _assert(y, O.linear(_np(x), _np(w), _np(bias), None, _NAME[dtype]), dtype, "linear")


@pytest.mark.parametrize("kind", ["dot", "simt"])
def test_linear_decode_shape_and_strided_weight(kind):
    torch.manual_seed(7)
    dtype = torch.float16
    x = torch.randn(1, 4096, device="cuda", dtype=dtype) * (4096**-0.5)
    w = torch.randn(1024, 4096, device="cuda", dtype=dtype) * (4096**-0.5)
    _assert(linear_decode(x, w, kind=kind), O.linear(_np(x), _np(w), None, None, "float16"), dtype, "linear")

    raw = torch.randn(128, 64, device="cuda", dtype=dtype)
    w_t = raw.t()
    assert not w_t.is_contiguous()
    x2 = torch.randn(4, 128, device="cuda", dtype=dtype) * (128**-0.5)
    row = torch.randn(4, 64, device="cuda", dtype=dtype)
    y = linear_decode(x2, w_t, row_add=row, kind=kind)
    _assert(y, O.linear(_np(x2), _np(w_t), None, _np(row), "float16"), dtype, "linear")


def test_linear_fallback_matches_cublas():
    torch.manual_seed(8)
    x = torch.randn(20, 32, device="cuda", dtype=torch.float16)
    w = torch.randn(48, 32, device="cuda", dtype=torch.float16)
    bias = torch.randn(48, device="cuda", dtype=torch.float16)
    y = linear_decode(x, w, bias)
    torch.testing.assert_close(y, F.linear(x, w, bias), rtol=0, atol=0)

    row = torch.randn(20, 48, device="cuda", dtype=torch.float16)
    fused = linear_decode(x, w, row_add=row)
    manual = F.linear(x, w) + row
    torch.testing.assert_close(fused, manual, rtol=1e-3, atol=1e-3)


def test_post_attn_mlp():
    torch.manual_seed(9)
    dtype = torch.float16
    hidden = 64
    inner = 128
    x = torch.randn(4, hidden, device="cuda", dtype=dtype)
    norm_w = torch.randn(hidden, device="cuda", dtype=dtype)
    w_gu = torch.randn(inner * 2, hidden, device="cuda", dtype=dtype) * (hidden**-0.5)
    w_down = torch.randn(hidden, inner, device="cuda", dtype=dtype) * (inner**-0.5)
    ref = O.post_attn_mlp(_np(x), _np(norm_w), _np(w_gu), _np(w_down), 1e-6, "float16")
    for kind in ("dot", "simt"):
        y = post_attn_mlp(x, norm_w, w_gu, w_down, kind=kind)
        _assert(y, ref, dtype, "linear")


def test_rejected_inputs():
    x = torch.randn(4, 16)
    w = torch.randn(16)
    with pytest.raises(ValueError, match="CUDA"):
        rms_norm(x, w)
    cuda = torch.randn(4, 16, device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="weight"):
        rms_norm(cuda, torch.randn(8, device="cuda", dtype=torch.float16))
    with pytest.raises(ValueError, match="even"):
        rope(
            torch.randn(2, 3, device="cuda", dtype=torch.float16),
            torch.randn(2, 3, device="cuda", dtype=torch.float16),
            torch.randn(2, 3, device="cuda", dtype=torch.float16),
        )


# ------------------------------------------------------------------ golden vectors
def _run_cuda(case):
    i = {k: to_torch(v) for k, v in case["inputs"].items()}
    p = case["params"]
    op = case["op"]
    if op == "rms_norm":
        x = i["x"]
        if p.get("layout") == "transposed":
            x = x.t().contiguous().t()  # same values, column-major storage
        return {"y": rms_norm(x, i["weight"], p["eps"])}
    if op == "add_rms_norm":
        r = i["residual"].clone()
        y, ro = add_rms_norm(i["x"], r, i["weight"], p["eps"], residual_out=r)
        return {"y": y, "residual_out": ro}
    if op == "swiglu":
        return {"y": swiglu(i["gate"], i["up"])}
    if op == "rope":
        x = i["x"]
        if p.get("layout") == "transposed":
            x = x.transpose(1, 2).contiguous().transpose(1, 2)
        return {"y": rope(x, i["cos"], i["sin"])}
    if op == "linear":
        w = i["weight"]
        if p.get("layout") == "transposed_weight":
            w = w.t().contiguous().t()
        return {"y": linear_decode(i["x"], w, i.get("bias"), row_add=i.get("row_add"), kind="dot")}
    if op == "post_attn_mlp":
        return {"y": post_attn_mlp(i["hidden"], i["norm_weight"], i["w_gate_up"], i["w_down"], p["eps"])}
    raise AssertionError(op)


_GOLDEN = load_golden()


@pytest.mark.parametrize("case", _GOLDEN, ids=[f"{c['id']}-{c['op']}-{c['dtype']}" for c in _GOLDEN])
def test_golden(case):
    """CUDA output vs the reference's own stored output: within the
    reference tolerance, and within 1 ulp of the activation dtype for the
    row/elementwise ops (the GEMV accumulates in a different order, so its
    rounded outputs may differ by a few ulp where cancellation is strong)."""
    dtype = torch.float16 if case["dtype"] == "float16" else torch.bfloat16
    got = _run_cuda(case)
    kind = "linear" if case["op"] in ("linear", "post_attn_mlp") else "pointwise"
    for name, (want, _) in case["outputs"].items():
        _assert(got[name], want, dtype, kind)
        if kind == "pointwise":
            d = O.ulp_distance(_np(got[name]), want, case["dtype"])
            assert d.max() <= 1, f"{name}: {d.max()} ulp"
            assert np.mean(d == 0) >= 0.99
