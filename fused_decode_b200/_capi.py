"""ctypes binding of the C ABI in ``include/fd_b200.h`` (``libfd_b200.so``),
and the loader of the compiled dispatch module ``_fastpath`` that calls the
same entry points from C++.

These are the only places Python reaches the native code.  Loading fails
loudly when either has not been built: there is no CPU or PyTorch fallback
behind these entry points.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_NAME = "libfd_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# fd_dtype
FD_F16, FD_BF16, FD_F32 = 0, 1, 2
# fd_kind
FD_KIND_DOT, FD_KIND_SIMT = 0, 1

_DTYPE_CODE = {torch.float16: FD_F16, torch.bfloat16: FD_BF16, torch.float32: FD_F32}

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_vp = ctypes.c_void_p
c_size = ctypes.c_size_t


class FdRows(ctypes.Structure):
    """``fd_rows``: a row grid (the reference's RowLayout, kernels.py:26-40)."""

    _fields_ = [
        ("ptr", c_vp),
        ("dtype", c_i32),
        ("_pad", c_i32),
        ("a", c_i64),
        ("b", c_i64),
        ("c", c_i64),
        ("sa", c_i64),
        ("sb", c_i64),
        ("sc", c_i64),
        ("col", c_i64),
        ("n", c_i64),
    ]


_P_ROWS = ctypes.POINTER(FdRows)

# name -> (restype, argtypes).  Every symbol declared in include/fd_b200.h.
SIGNATURES: dict[str, tuple] = {
    "fd_status_string": (ctypes.c_char_p, [c_i32]),
    "fd_device_sm_count": (c_i32, []),
    "fd_rms_out": (c_i32, [_P_ROWS, _P_ROWS, c_vp, c_i32, c_i64, _P_ROWS, _P_ROWS, c_f32, c_vp]),
    "fd_swiglu_out": (c_i32, [_P_ROWS, _P_ROWS, _P_ROWS, c_vp]),
    "fd_rope_out": (c_i32, [_P_ROWS, _P_ROWS, _P_ROWS, _P_ROWS, c_vp]),
    "fd_linear_workspace_bytes": (c_size, [c_i32, c_i64, c_i64]),
    "fd_workspace_status_offset": (c_size, []),
    "fd_linear_out": (
        c_i32,
        [
            c_vp, c_i64, c_i64,          # x, sxm, sxk
            c_vp, c_i64, c_i64,          # w, swn, swk
            c_vp, c_i32, c_i64,          # bias, bias_dtype, sbias
            c_vp, c_i32, c_i64, c_i64,   # row_add, ra_dtype, srm, srn
            c_vp, c_i64, c_i64,          # y, sym, syn
            c_i32, c_i32, c_i64, c_i64, c_i32,  # dtype, m, n, k, kind
            c_vp, c_size, c_vp,          # workspace, bytes, stream
        ],
    ),
    "fd_linear_noalloc_scratch_bytes": (c_size, []),
    "fd_linear_noalloc_status": (c_i32, [ctypes.POINTER(c_i32), c_vp]),
    "fd_linear_noalloc_reset": (c_i32, [c_vp]),
    "fd_linear_out_noalloc": (
        c_i32,
        [
            c_vp, c_i64, c_i64,          # x, sxm, sxk
            c_vp, c_i64, c_i64,          # w, swn, swk
            c_vp, c_i32, c_i64,          # bias, bias_dtype, sbias
            c_vp, c_i32, c_i64, c_i64,   # row_add, ra_dtype, srm, srn
            c_vp, c_i64, c_i64,          # y, sym, syn
            c_i32, c_i32, c_i64, c_i64, c_i32,  # dtype, m, n, k, kind
            c_vp,                        # stream
        ],
    ),
    "fd_tp_exchange_bytes": (c_size, [c_i32, c_i32, c_i64]),
    "fd_tp_exchange_alloc": (c_i32, [c_i32, c_i32, c_i64, ctypes.POINTER(c_vp)]),
    "fd_tp_exchange_free": (c_i32, [c_vp]),
    "fd_tp_exchange_handle": (c_i32, [c_vp, c_vp]),
    "fd_tp_exchange_open": (c_i32, [c_vp, ctypes.POINTER(c_vp)]),
    "fd_tp_exchange_close": (c_i32, [c_vp]),
    "fd_post_attn_mlp_tp_out": (
        c_i32,
        [
            c_vp, c_vp, c_i32,           # hidden, norm_w, norm_dtype
            c_vp, c_i64, c_vp, c_i64,    # w_gate_up, s_gu, w_down, s_down
            c_vp, c_i32, c_i32, c_i64, c_i64,  # out, dtype, m, h, i
            c_f32, c_i32, c_i32, c_i32,  # eps, kind, rank, world
            c_vp, c_i32,                 # exchange (void* const*), m_max
            c_vp, c_size, c_vp,          # workspace, bytes, stream
        ],
    ),
    "fd_post_attn_mlp_workspace_bytes": (c_size, [c_i32, c_i64, c_i64]),
    "fd_post_attn_mlp_out": (
        c_i32,
        [
            c_vp, c_vp, c_i32,           # hidden, norm_w, norm_dtype
            c_vp, c_i64, c_vp, c_i64,    # w_gate_up, s_gu, w_down, s_down
            c_vp, c_i32, c_i32,          # out, out_dtype, dtype
            c_i32, c_i64, c_i64,         # m, h, i
            c_f32, c_i32, c_i32,         # eps, kind, add_residual
            c_vp, c_size, c_vp,          # workspace, bytes, stream
        ],
    ),
    "fd_mlp_gate_up_out": (
        c_i32,
        [
            c_vp, c_vp, c_i32,           # hidden, norm_w, norm_dtype
            c_vp, c_i64, c_vp, c_i32,    # w_gate_up, s_gu, mid, dtype
            c_i32, c_i64, c_i64,         # m, h, i
            c_f32, c_i32,                # eps, kind
            c_vp, c_size, c_vp,          # workspace, bytes, stream
        ],
    ),
    "fd_post_attn_mlp_stack_launches": (c_i32, [c_i32, c_i32, c_i32, c_i64, c_i64, c_i32]),
    "fd_post_attn_mlp_layer_launches": (c_i32, [c_i32, c_i64, c_i64, c_i32, c_i32, c_i32]),
    "fd_post_attn_mlp_tp_stack_launches": (c_i32, [c_i32, c_i32, c_i32, c_i64, c_i64, c_i32]),
    "fd_post_attn_mlp_tp_stack_out": (
        c_i32,
        [
            c_vp, c_i32,                 # hidden, layers
            c_vp, c_i32,                 # norm_w (host array), norm_dtype
            c_vp, c_i64, c_vp, c_i64,    # w_gate_up (host array), s_gu, w_down (host array), s_down
            c_vp, c_i32, c_i32, c_i64, c_i64,  # out, dtype, m, h, i
            c_f32, c_i32, c_i32, c_i32,  # eps, kind, rank, world
            c_vp, c_i32,                 # exchange (void* const*), m_max
            c_vp, c_size, c_vp,          # workspace, bytes, stream
        ],
    ),
    "fd_post_attn_mlp_stack_out": (
        c_i32,
        [
            c_vp, c_i32,                 # hidden, layers
            c_vp, c_i32,                 # norm_w[], norm_dtype
            c_vp, c_i64, c_vp, c_i64,    # w_gate_up[], s_gu, w_down[], s_down
            c_vp, c_i32, c_i32,          # out, dtype, m
            c_i64, c_i64, c_f32, c_i32,  # h, i, eps, kind
            c_vp, c_size, c_vp,          # workspace, bytes, stream
        ],
    ),
    "fd_residual_add_out": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i64, c_vp]),
    "fd_copy": (c_i32, [c_vp, c_vp, c_size, c_vp]),
    "fd_triad": (c_i32, [c_vp, c_vp, c_vp, c_i64, c_i32, c_f32, c_vp]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load ``libfd_b200.so`` once and bind every signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_NAME} is not built ({LIB_PATH} missing). "
                "Build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "or `python -m fused_decode_b200.build`."
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


_fast = None


def fast():
    """The compiled dispatch module ``_fastpath`` (csrc/fd_fastpath.cpp), loaded
    once; like ``load()`` it fails loudly when it has not been built."""
    global _fast
    if _fast is None:
        load()
        try:
            from fused_decode_b200 import _fastpath
        except ImportError as exc:
            raise RuntimeError(
                "the _fastpath extension is not built (or does not load): "
                "build it with `python -m fused_decode_b200.build`"
            ) from exc
        _fast = _fastpath
    return _fast


def fast_or_none():
    """``fast()``, or None when either native module is missing.  The
    operators use this to offer a call to the compiled path first; when it is
    absent their Python path still fails loudly at the launch (``load()``)."""
    if _fast is not None:
        return _fast
    try:
        return fast()
    except RuntimeError:
        return None


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().fd_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {msg} (status {status})")


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr_array(ptrs) -> ctypes.Array:
    """A host array of device pointers (``const void* const*``)."""
    return (c_vp * len(ptrs))(*ptrs)


def rows(layout) -> FdRows:
    """Pack a kernels.RowLayout into an fd_rows struct."""
    t = layout.tensor
    return FdRows(
        t.data_ptr(),
        dtype_code(t.dtype),
        0,
        layout.a,
        layout.b,
        layout.c,
        layout.sa,
        layout.sb,
        layout.sc,
        layout.col,
        layout.n,
    )
