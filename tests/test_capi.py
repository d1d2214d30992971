"""The C ABI boundary (include/fd_b200.h <-> libfd_b200.so).

CPU part: the library loads and exports every symbol the header declares, and
the Python binding covers exactly that set.  GPU part: direct calls with raw
device pointers, status codes for rejected arguments, and parity of a direct
call with the oracle.
"""

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fd_b200.h")


def _declared() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(fd_[a-z0-9_]+)\s*\(", text))


def test_header_declares_entry_points():
    names = _declared()
    for want in ("fd_rms_out", "fd_swiglu_out", "fd_rope_out", "fd_linear_out",
                 "fd_post_attn_mlp_out", "fd_copy", "fd_triad"):
        assert want in names


def test_library_exports_every_declared_symbol():
    from fused_decode_b200 import _capi

    lib = ctypes.CDLL(_capi.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in fd_b200.h but not exported"


def test_binding_covers_header():
    from fused_decode_b200 import _capi

    assert set(_capi.SIGNATURES) == _declared()


def test_status_strings_without_gpu():
    from fused_decode_b200 import _capi

    lib = _capi.load()
    assert lib.fd_status_string(0) == b"ok"
    assert lib.fd_status_string(3) == b"workspace missing or too small"


def test_fd_rows_layout_matches_header():
    from fused_decode_b200 import _capi

    # void* + 2 x int32 + 8 x int64
    assert ctypes.sizeof(_capi.FdRows) == 8 + 8 + 8 * 8


# ------------------------------------------------------------------ GPU
@pytest.mark.gpu
def test_direct_linear_call_and_status_codes():
    import torch

    from fused_decode_b200 import _capi
    from oracle import fd_oracle as O

    lib = _capi.load()
    m, n, k = 4, 300, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    need = lib.fd_linear_workspace_bytes(m, n, k)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def call(wsp, wsb, mm=m, dtype=_capi.FD_BF16, kind=_capi.FD_KIND_DOT):
        return lib.fd_linear_out(x.data_ptr(), k, 1, w.data_ptr(), k, 1, None, 0, 0, None, 0, 0, 0,
                                 y.data_ptr(), n, 1, dtype, mm, n, k, kind, wsp, wsb, stream)

    assert call(ws.data_ptr(), need) == 0
    torch.cuda.synchronize()
    ref = O.linear(x.float().cpu().numpy(), w.float().cpu().numpy(), None, None, "bfloat16")
    torch.testing.assert_close(y.float().cpu(), torch.from_numpy(ref), rtol=1e-2, atol=1e-2)
    assert call(ws.data_ptr(), need - 1) == 3       # FD_ERR_WORKSPACE
    assert call(None, 0) == 3
    assert call(ws.data_ptr(), need, mm=17) == 4    # FD_ERR_UNSUPPORTED (M > 16)
    assert call(ws.data_ptr(), need, dtype=2) == 1  # FD_ERR_ARG (f32 activations)
    assert call(ws.data_ptr(), need, kind=7) == 1   # FD_ERR_ARG (bad kind)


@pytest.mark.gpu
def test_direct_copy_and_triad():
    import torch

    from fused_decode_b200 import kernels as K

    a = torch.randn(1 << 20, device="cuda", dtype=torch.float16)
    b = torch.randn(1 << 20, device="cuda", dtype=torch.float16)
    c = torch.empty_like(a)
    K.launch_copy(c, a)
    assert torch.equal(c, a)
    K.launch_triad(a, b, c, 1.25)
    torch.testing.assert_close(c.float(), a.float() + b.float() * 1.25, rtol=1e-3, atol=1e-3)
    # odd byte counts and misaligned pointers take the byte path
    src = torch.arange(1001, device="cuda", dtype=torch.uint8)
    dst = torch.zeros(1001, device="cuda", dtype=torch.uint8)
    K.launch_copy(dst[1:], src[1:])
    assert torch.equal(dst[1:], src[1:])


def test_layer_launch_counts_without_gpu(monkeypatch):
    """Kernel launches one post_attn_mlp layer enqueues -- a host-side plan,
    so no GPU is needed: two (gate/up, down); three where the gate/up stage
    streams the normalised rows because the resident batch would leave its
    shared-memory ring under 4 stages (8B hidden width above 10 rows, 9 with
    an fp32 norm weight; 70B hidden width above 4); one more for the
    tensor-parallel rank sum, unless FD_TP_FOLD=1 folds it into the down
    projection (dot consumers only).  FD_GATEUP_STREAM forces either mode."""
    import torch

    from fused_decode_b200 import _capi

    lib = _capi.load()
    bf, f32 = _capi.dtype_code(torch.bfloat16), _capi.dtype_code(torch.float32)
    dot, simt = _capi.FD_KIND_DOT, _capi.FD_KIND_SIMT
    monkeypatch.delenv("FD_GATEUP_STREAM", raising=False)
    monkeypatch.delenv("FD_TP_FOLD", raising=False)

    def n(m, h, nd=bf, kind=dot, tp=0):
        return lib.fd_post_attn_mlp_layer_launches(m, h, 14336, nd, kind, tp)

    assert [n(m, 4096) for m in (1, 8, 10, 11, 16)] == [2, 2, 2, 3, 3]
    assert [n(m, 4096, nd=f32) for m in (9, 10)] == [2, 3]
    assert [n(m, 8192) for m in (1, 4, 5, 8, 16)] == [2, 2, 3, 3, 3]
    assert n(1, 4096, tp=1) == 3 and n(8, 8192, tp=1) == 4
    monkeypatch.setenv("FD_TP_FOLD", "1")
    assert n(1, 4096, tp=1) == 2 and n(8, 8192, tp=1) == 3
    assert n(1, 4096, kind=simt, tp=1) == 3  # the fold has dot instantiations only
    monkeypatch.delenv("FD_TP_FOLD")
    monkeypatch.setenv("FD_GATEUP_STREAM", "1")
    assert n(1, 4096) == 3
    monkeypatch.setenv("FD_GATEUP_STREAM", "0")
    assert n(16, 4096) == 2
    assert n(0, 4096) == 0
