"""Edge cases of the row operators on the GPU, against the oracle: empty
batches, five-dimensional inputs (made contiguous first, as the reference's
row_layout does), outputs written into non-contiguous views, and a 1-row
batch.  (Negative strides, which row_layout also copies away, cannot be made
with PyTorch tensors; tests/test_row_layout_cpu.py covers the layout side.)  Tolerance: the reference's table
(tests/test_ops.py:27-35 of the reference): atol = rtol = 1e-2 for these
fp16/bf16 pointwise ops."""

import numpy as np
import pytest
import torch

from oracle import fd_oracle as O

pytestmark = pytest.mark.gpu

import fused_decode_b200 as fd  # noqa: E402

TOL = {"rtol": 1e-2, "atol": 1e-2}
BF, F16 = torch.bfloat16, torch.float16


def _np(t):
    return t.detach().float().cpu().numpy()


def _close(actual, expected):
    torch.testing.assert_close(actual.float().cpu(), torch.from_numpy(np.ascontiguousarray(expected)), **TOL)


def test_empty_batches():
    w = torch.randn(64, device="cuda", dtype=BF)
    x = torch.empty(0, 64, device="cuda", dtype=BF)
    assert fd.rms_norm(x, w).shape == (0, 64)
    y, r = fd.add_rms_norm(x, torch.empty_like(x), w)
    assert y.shape == r.shape == (0, 64)
    assert fd.swiglu(x, x).shape == (0, 64)
    q = torch.empty(1, 0, 4, 64, device="cuda", dtype=F16)
    cs = torch.empty(0, 1, 64, device="cuda", dtype=F16)
    assert fd.rope(q, cs, cs).shape == q.shape
    wl = torch.randn(32, 64, device="cuda", dtype=BF)
    assert fd.linear_decode(x, wl).shape == (0, 32)


def test_five_dims_and_reordered_inputs():
    torch.manual_seed(3)
    x5 = torch.randn(2, 3, 2, 2, 128, device="cuda", dtype=BF)
    w = torch.randn(128, device="cuda", dtype=BF)
    _close(fd.rms_norm(x5, w, 1e-5), O.rms_norm(_np(x5), _np(w), 1e-5, "bfloat16"))
    xf = torch.randn(6, 256, device="cuda", dtype=F16).flip(0)
    wf = torch.randn(256, device="cuda", dtype=F16)
    _close(fd.rms_norm(xf, wf, 1e-5), O.rms_norm(_np(xf), _np(wf), 1e-5, "float16"))
    g = torch.randn(4, 512, device="cuda", dtype=BF).flip(1)
    u = torch.randn(4, 512, device="cuda", dtype=BF)
    _close(fd.swiglu(g, u), O.swiglu(_np(g), _np(u), "bfloat16"))


def test_out_into_views_and_single_row():
    torch.manual_seed(4)
    x = torch.randn(5, 384, device="cuda", dtype=F16)
    w = torch.randn(384, device="cuda", dtype=F16)
    big = torch.zeros(5, 512, device="cuda", dtype=F16)
    view = big[:, 64:448]  # a non-contiguous output view
    fd.rms_norm(x, w, 1e-5, out=view)
    _close(view, O.rms_norm(_np(x), _np(w), 1e-5, "float16"))
    assert torch.count_nonzero(big[:, :64]) == 0 and torch.count_nonzero(big[:, 448:]) == 0
    x1 = torch.randn(1, 8192, device="cuda", dtype=BF)
    r1 = torch.randn(1, 8192, device="cuda", dtype=BF)
    w1 = torch.randn(8192, device="cuda", dtype=torch.float32)
    y, s = fd.add_rms_norm(x1, r1, w1, 1e-5)
    ry, rs = O.add_rms_norm(_np(x1), _np(r1), _np(w1), 1e-5, "bfloat16")
    _close(y, ry)
    _close(s, rs)
