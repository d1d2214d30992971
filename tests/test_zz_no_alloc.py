"""fd_linear_out_noalloc: the GEMV with its scratch in static device memory.

Calls the entry point through the C ABI (ctypes) twice in a row and compares
each result with fd_linear_out given an ordinary caller workspace, on the same
inputs.  Tolerance: BASELINE's atol = rtol = 1e-2 (the two entries run the same
kernels, so in practice the outputs are identical).  Runs last in the suite
and also passes on its own in a fresh process: the first call on the device
does the scratch set-up.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

from fused_decode_b200 import _capi  # noqa: E402
from fused_decode_b200 import kernels as K  # noqa: E402

TOL = {"rtol": 1e-2, "atol": 1e-2}


def _args(x, w, bias, row_add, y, kind):
    m, k = x.shape
    n = w.shape[0]
    if bias is not None:
        b = (bias.data_ptr(), _capi.dtype_code(bias.dtype), int(bias.stride(0)))
    else:
        b = (None, 0, 0)
    if row_add is not None:
        ra = (row_add.data_ptr(), _capi.dtype_code(row_add.dtype), int(row_add.stride(0)), int(row_add.stride(1)))
    else:
        ra = (None, 0, 0, 0)
    return (
        x.data_ptr(), int(x.stride(0)), int(x.stride(1)),
        w.data_ptr(), int(w.stride(0)), int(w.stride(1)),
        *b, *ra,
        y.data_ptr(), int(y.stride(0)), int(y.stride(1)),
        _capi.dtype_code(x.dtype), m, n, k,
        _capi.FD_KIND_DOT if kind == "dot" else _capi.FD_KIND_SIMT,
    )


@pytest.mark.parametrize("kind", ["dot", "simt"])
@pytest.mark.parametrize("m,n,k,extras", [(1, 4096, 14336, False), (8, 14336, 4096, True), (3, 1000, 320, True)])
def test_noalloc_matches_workspace_entry(kind, m, n, k, extras):
    lib = _capi.load()
    assert lib.fd_linear_noalloc_scratch_bytes() >= lib.fd_linear_workspace_bytes(m, n, k)
    g = torch.Generator(device="cuda").manual_seed(1000 + m)
    dt = torch.bfloat16
    x = torch.randn(m, k, device="cuda", dtype=dt, generator=g)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(dt)
    bias = (torch.randn(n, device="cuda", generator=g) * 0.02).to(dt) if extras else None
    row_add = torch.randn(m, n, device="cuda", dtype=dt, generator=g) if extras else None
    stream = _capi.stream_of(x)

    y_ws = torch.empty(m, n, device="cuda", dtype=dt)
    ws = K.WORKSPACES.get(x.device, lib.fd_linear_workspace_bytes(m, n, k))
    st = lib.fd_linear_out(*_args(x, w, bias, row_add, y_ws, kind), ws.data_ptr(), ws.numel(), stream)
    assert st == 0, lib.fd_status_string(st)

    for _ in range(2):  # two calls in a row: the scratch is left ready for the next call
        y = torch.full((m, n), float("nan"), device="cuda", dtype=dt)
        st = lib.fd_linear_out_noalloc(*_args(x, w, bias, row_add, y, kind), stream)
        assert st == 0, lib.fd_status_string(st)
        torch.cuda.synchronize()
        torch.testing.assert_close(y.float(), y_ws.float(), **TOL)


def test_noalloc_rejects_bad_arguments():
    lib = _capi.load()
    x = torch.randn(17, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(32, 64, device="cuda", dtype=torch.float16)
    y = torch.empty(17, 32, device="cuda", dtype=torch.float16)
    st = lib.fd_linear_out_noalloc(*_args(x, w, None, None, y, "dot"), ctypes.c_void_p(None))
    assert st != 0  # M > 16 is outside the GEMV family
