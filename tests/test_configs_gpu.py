"""Parity of the standalone operators at the benchmark configurations' full shapes.

These are the shapes the benchmark times, where the vector kernels take
different paths than at the small test shapes (multi-row CTAs, one-wave
grid-stride loops, 32-bit row splits):

* add_rms_norm: x, residual [8192, 4096] fp16 ~ N(0, 1), weight = 1 + 0.1 N(0, 1),
  eps = 1e-5, ``residual_out=residual`` (in place: the same storage comes back);
* rms_norm: [8192, 4096] and [1, 4096];
* swiglu: gate, up [2048, 14336] and [1, 14336], fp16 and bf16;
* rope: x [1, 2048, 32, 128] and [1, 1, 32, 128] fp16, cos/sin built from
  theta = 500000 for positions 0..2047, passed as [T, 1, 128] (broadcast over
  the heads).

Each output is checked against the CPU oracle (a numpy restatement of the
reference's reference.py, pinned by tests/test_oracle_golden.py) at the parity
bar atol = rtol = 1e-2, with exact shape, stride and dtype equality.
"""

import numpy as np
import pytest
import torch

import fused_decode_b200 as fd
from oracle import fd_oracle as O

pytestmark = pytest.mark.gpu

TOL = {"rtol": 1e-2, "atol": 1e-2}
H, I = 4096, 14336
_NAME = {torch.float16: O.F16, torch.bfloat16: O.BF16}


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.fail("CUDA GPU required for -m gpu tests")
    from fused_decode_b200 import _capi

    _capi.load()


def _gen(seed=0):
    return torch.Generator(device="cuda").manual_seed(seed)


def _np(t):
    return t.detach().float().cpu().numpy()


def _check(actual, expected_np, like, what):
    assert actual.shape == like.shape, what
    assert actual.dtype == like.dtype, what
    assert actual.stride() == torch.empty(like.shape).stride(), what  # fresh outputs are contiguous
    expected = torch.from_numpy(np.ascontiguousarray(expected_np))
    torch.testing.assert_close(actual.float().cpu(), expected, **TOL, msg=lambda s: f"{what}: {s}")


def _rope_tables(positions, dim, dtype, theta=500000.0, first=0):
    inv = theta ** (-torch.arange(0, dim, 2, dtype=torch.float32, device="cuda") / dim)
    pos = torch.arange(first, first + positions, dtype=torch.float32, device="cuda")
    f = torch.outer(pos, inv)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(dtype).view(positions, 1, dim), emb.sin().to(dtype).view(positions, 1, dim)


def test_add_rms_norm_8192x4096_fp16_in_place():
    g = _gen(0)
    dt = torch.float16
    x = torch.randn(8192, H, device="cuda", dtype=dt, generator=g)
    res = torch.randn(8192, H, device="cuda", dtype=dt, generator=g)
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(dt)
    y_ref, r_ref = O.add_rms_norm(_np(x), _np(res), _np(w), 1e-5, O.F16)
    ptr = res.data_ptr()
    y, r = fd.add_rms_norm(x, res, w, 1e-5, residual_out=res)
    torch.cuda.synchronize()
    assert r.data_ptr() == ptr and res.data_ptr() == ptr  # written in place
    _check(y, y_ref, x, "add_rms_norm out")
    _check(r, r_ref, x, "add_rms_norm residual_out")


@pytest.mark.parametrize("rows", [8192, 1])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rms_norm_config_shapes(rows, dtype):
    g = _gen(1)
    x = torch.randn(rows, H, device="cuda", dtype=dtype, generator=g)
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(dtype)
    _check(fd.rms_norm(x, w, 1e-5), O.rms_norm(_np(x), _np(w), 1e-5, _NAME[dtype]), x, f"rms_norm {rows}")


@pytest.mark.parametrize("rows", [2048, 1])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_swiglu_config_shapes(rows, dtype):
    g = _gen(2)
    gate = torch.randn(rows, I, device="cuda", dtype=dtype, generator=g)
    up = torch.randn(rows, I, device="cuda", dtype=dtype, generator=g)
    _check(fd.swiglu(gate, up), O.swiglu(_np(gate), _np(up), _NAME[dtype]), gate, f"swiglu {rows}")


@pytest.mark.parametrize("tokens,first", [(2048, 0), (1, 0), (1, 2047)])
def test_rope_theta_tables(tokens, first):
    """x [1, T, 32, 128] fp16 with theta = 500000 cos/sin as [T, 1, 128]."""
    g = _gen(3)
    dt = torch.float16
    x = torch.randn(1, tokens, 32, 128, device="cuda", dtype=dt, generator=g)
    cos, sin = _rope_tables(tokens, 128, dt, first=first)
    ref = O.rope(_np(x), _np(cos), _np(sin), O.F16)
    _check(fd.rope(x, cos, sin), ref, x, f"rope T={tokens} from {first}")


def test_rope_bf16_full_length():
    g = _gen(4)
    dt = torch.bfloat16
    x = torch.randn(1, 2048, 32, 128, device="cuda", dtype=dt, generator=g)
    cos, sin = _rope_tables(2048, 128, dt)
    _check(fd.rope(x, cos, sin), O.rope(_np(x), _np(cos), _np(sin), O.BF16), x, "rope bf16")
