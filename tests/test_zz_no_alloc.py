"""fd_linear_out_noalloc: the GEMV with its scratch in static device memory.

For callers that cannot hand the library device memory (no allocator of
their own, or a memory plan frozen after start-up).  Calls the entry point
through the C ABI (ctypes) twice in a row and checks each result against the
CPU oracle at the parity bar atol = rtol = 1e-2, and against fd_linear_out
given an ordinary caller workspace (the same kernels, so the same bits).
After every call the scratch's status word must read zero; a reset must
leave a scratch that gives the same results.  Runs last in the suite and
also passes on its own in a fresh process: the first call on the device does
the scratch set-up.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

from fused_decode_b200 import _capi  # noqa: E402
from fused_decode_b200 import kernels as K  # noqa: E402
from oracle import fd_oracle as O  # noqa: E402

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


def _np(t):
    return t.detach().float().cpu().numpy()


def _status(lib, stream) -> int:
    v = ctypes.c_int32(-1)
    st = lib.fd_linear_noalloc_status(ctypes.byref(v), stream)
    assert st == 0, lib.fd_status_string(st)
    return v.value


def _inputs(m, n, k, extras, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dt = torch.bfloat16
    x = torch.randn(m, k, device="cuda", dtype=dt, generator=g)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(dt)
    bias = (torch.randn(n, device="cuda", generator=g) * 0.02).to(dt) if extras else None
    row_add = torch.randn(m, n, device="cuda", dtype=dt, generator=g) if extras else None
    return x, w, bias, row_add


def _oracle(x, w, bias, row_add):
    return O.linear(_np(x), _np(w), None if bias is None else _np(bias), None if row_add is None else _np(row_add),
                    O.BF16)


@pytest.mark.parametrize("kind", ["dot", "simt"])
@pytest.mark.parametrize("m,n,k,extras", [(1, 4096, 14336, False), (8, 14336, 4096, True), (3, 1000, 320, True)])
def test_noalloc_matches_oracle_and_workspace_entry(kind, m, n, k, extras):
    lib = _capi.load()
    assert lib.fd_linear_noalloc_scratch_bytes() >= lib.fd_linear_workspace_bytes(m, n, k)
    x, w, bias, row_add = _inputs(m, n, k, extras, 1000 + m)
    stream = _capi.stream_of(x)
    ref = torch.from_numpy(_oracle(x, w, bias, row_add))

    y_ws = torch.empty(m, n, device="cuda", dtype=x.dtype)
    ws = K.WORKSPACES.get(x.device, lib.fd_linear_workspace_bytes(m, n, k))
    st = lib.fd_linear_out(*_args(x, w, bias, row_add, y_ws, kind), ws.data_ptr(), ws.numel(), stream)
    assert st == 0, lib.fd_status_string(st)

    for _ in range(2):  # two calls in a row: the scratch is left ready for the next call
        y = torch.full((m, n), float("nan"), device="cuda", dtype=x.dtype)
        st = lib.fd_linear_out_noalloc(*_args(x, w, bias, row_add, y, kind), stream)
        assert st == 0, lib.fd_status_string(st)
        assert _status(lib, stream) == 0
        torch.testing.assert_close(y.float().cpu(), ref, **TOL)
        assert torch.equal(y, y_ws)


def test_noalloc_and_workspace_calls_back_to_back():
    """A workspace call and a no-alloc call queued on one stream with nothing
    between them: the two scratches are separate, both results are right."""
    lib = _capi.load()
    m, n, k = 4, 4096, 4096
    x, w, bias, row_add = _inputs(m, n, k, True, 7)
    stream = _capi.stream_of(x)
    ref = torch.from_numpy(_oracle(x, w, bias, row_add))
    ws = K.WORKSPACES.get(x.device, lib.fd_linear_workspace_bytes(m, n, k))
    ys = [torch.full((m, n), float("nan"), device="cuda", dtype=x.dtype) for _ in range(4)]
    for j, y in enumerate(ys):
        if j % 2 == 0:
            st = lib.fd_linear_out(*_args(x, w, bias, row_add, y, "dot"), ws.data_ptr(), ws.numel(), stream)
        else:
            st = lib.fd_linear_out_noalloc(*_args(x, w, bias, row_add, y, "dot"), stream)
        assert st == 0, lib.fd_status_string(st)
    assert _status(lib, stream) == 0
    for y in ys:
        torch.testing.assert_close(y.float().cpu(), ref, **TOL)
        assert torch.equal(y, ys[0])


def test_noalloc_reset_then_calls():
    """fd_linear_noalloc_reset zeroes the counters and status on the stream;
    the calls after it give the oracle's results and leave the status at 0."""
    lib = _capi.load()
    m, n, k = 2, 14336, 4096
    x, w, _, _ = _inputs(m, n, k, False, 11)
    stream = _capi.stream_of(x)
    ref = torch.from_numpy(_oracle(x, w, None, None))
    st = lib.fd_linear_noalloc_reset(stream)
    assert st == 0, lib.fd_status_string(st)
    assert _status(lib, stream) == 0
    for _ in range(2):
        y = torch.full((m, n), float("nan"), device="cuda", dtype=x.dtype)
        st = lib.fd_linear_out_noalloc(*_args(x, w, None, None, y, "dot"), stream)
        assert st == 0, lib.fd_status_string(st)
        torch.testing.assert_close(y.float().cpu(), ref, **TOL)
        st = lib.fd_linear_noalloc_reset(stream)
        assert st == 0, lib.fd_status_string(st)
    assert _status(lib, stream) == 0


def test_noalloc_rejects_bad_arguments():
    lib = _capi.load()
    x = torch.randn(17, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(32, 64, device="cuda", dtype=torch.float16)
    y = torch.empty(17, 32, device="cuda", dtype=torch.float16)
    st = lib.fd_linear_out_noalloc(*_args(x, w, None, None, y, "dot"), ctypes.c_void_p(None))
    assert st != 0  # M > 16 is outside the GEMV family
    assert lib.fd_linear_noalloc_status(None, ctypes.c_void_p(None)) != 0  # no place to put the status
