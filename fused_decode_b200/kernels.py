"""Launchers: the seam between the operator API and the sm_100a kernels.

Same names, argument order and preconditions as the reference launcher layer
(``src/fused_decode/kernels.py``): every launcher takes preallocated outputs and
returns ``None``.  Each one packs tensors into the C ABI of
``include/fd_b200.h`` and launches on PyTorch's current stream; none of them
synchronises the host, so all of them can be captured in a CUDA graph.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from fused_decode_b200 import _capi

# Default geometry of the stream-K GEMV (csrc/fd_stream.cuh): weight rows per
# block, columns per pipeline step (two 64-column TMA boxes), consumer warps
# per CTA, shared-memory ring stages.  The library may shed ring stages when a
# batch's activation rows need the shared memory; FD_GEMV_GEOMETRY overrides
# producers, boxes and stages for tuning.
GEMV_BLOCK_ROWS = 128
GEMV_K_STEP = 128
GEMV_WARPS = 8
GEMV_STAGES = 4
GEMV_MAX_M = 16


@dataclass(frozen=True)
class RowLayout:
    """Up to three leading dims plus the row (reference kernels.py:26-40)."""

    tensor: torch.Tensor
    a: int
    b: int
    c: int
    sa: int
    sb: int
    sc: int
    col: int
    n: int

    @property
    def rows(self) -> int:
        return self.a * self.b * self.c


def row_layout(t: torch.Tensor) -> RowLayout:
    """Describe ``t`` as a grid of rows over its last dimension.

    Mirrors reference kernels.py:43-70: leading dimensions are right-aligned
    into (a, b, c); tensors with more than four dimensions, or with a negative
    stride, are made contiguous first.
    """
    if t.ndim == 0:
        raise ValueError("expected a tensor with a last dimension")
    if any(s < 0 for s in t.stride()):
        t = t.contiguous()
    n = int(t.shape[-1])
    if t.ndim > 4:
        t = t.contiguous().reshape(-1, n)
    if t.ndim == 1:
        return RowLayout(t, 1, 1, 1, 0, 0, 0, int(t.stride(0)), n)
    lead = t.ndim - 1
    sizes = [1] * (3 - lead) + [int(s) for s in t.shape[:-1]]
    strides = [0] * (3 - lead) + [int(s) for s in t.stride()[:-1]]
    return RowLayout(t, *sizes, *strides, int(t.stride(-1)), n)


def _same_grid(left: RowLayout, right: RowLayout, what: str) -> None:
    if (left.a, left.b, left.c, left.n) != (right.a, right.b, right.c, right.n):
        raise ValueError(f"{what} cannot be indexed with the same row grid as the input")


def _runnable(layout: RowLayout) -> bool:
    return layout.rows > 0 and layout.n > 0


def _write_back(layout: RowLayout, target: torch.Tensor) -> None:
    """A >4-D non-contiguous output was laid out in a temporary; copy it home."""
    if layout.tensor.data_ptr() != target.data_ptr():
        target.copy_(layout.tensor.view(target.shape))


# ------------------------------------------------------------------ workspace
class _WorkspaceCache:
    """One zero-initialised scratch buffer per (device, stream).

    The buffers are held by the compiled dispatch module (``_fastpath``), so
    the Python launchers and the compiled fast path share them.  The split-K
    kernels leave their counters at zero when they finish, so a buffer is
    zero-filled only when it is first allocated or grown.  Launches that share
    a buffer must be stream-ordered, which the per-stream key guarantees.
    """

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        index = device.index if device.index is not None else torch.cuda.current_device()
        return _capi.fast().workspace(index, int(nbytes))

    def clear(self) -> None:
        _capi.fast().clear_workspaces()

    def status(self) -> dict:
        """Error bits of every cached workspace (synchronises the device).

        Non-zero means a kernel's bounded shared-memory pipeline wait expired
        (1: consumer, 2: producer) or a tensor-parallel exchange wait expired
        (8), and that output is not valid.
        """
        off = _capi.load().fd_workspace_status_offset()
        out = {}
        for key, buf in _capi.fast().workspaces():
            if buf.numel() >= off + 4:
                out[key] = int(buf[off:off + 4].view(torch.int32).item())
        return out


WORKSPACES = _WorkspaceCache()


# ------------------------------------------------------------------ RMSNorm
def rms_out(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    out: torch.Tensor,
    residual: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
) -> None:
    """RMSNorm / fused add+RMSNorm into ``out`` (reference kernels.py:343-414)."""
    lx = row_layout(x)
    ly = row_layout(out)
    _same_grid(lx, ly, "out")
    lr = row_layout(residual) if residual is not None else None
    lro = row_layout(residual_out) if residual_out is not None else None
    if lr is not None:
        _same_grid(lx, lr, "residual")
    if lro is not None:
        _same_grid(lx, lro, "residual_out")
    if not _runnable(lx):
        return
    lib = _capi.load()
    rx, ry = _capi.rows(lx), _capi.rows(ly)
    rr = _capi.rows(lr) if lr is not None else None
    rro = _capi.rows(lro) if lro is not None else None
    status = lib.fd_rms_out(
        rx,
        rr,
        weight.data_ptr(),
        _capi.dtype_code(weight.dtype),
        int(weight.stride(0)),
        ry,
        rro,
        float(eps),
        _capi.stream_of(x),
    )
    _capi.check(status, "fd_rms_out")
    _write_back(ly, out)
    if lro is not None:
        _write_back(lro, residual_out)


# ------------------------------------------------------------------ SwiGLU
def swiglu_out(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> None:
    """``out = silu(gate) * up`` (reference kernels.py:456-487)."""
    lg, lu, ly = row_layout(gate), row_layout(up), row_layout(out)
    _same_grid(lg, lu, "up")
    _same_grid(lg, ly, "out")
    if not _runnable(lg):
        return
    lib = _capi.load()
    status = lib.fd_swiglu_out(_capi.rows(lg), _capi.rows(lu), _capi.rows(ly), _capi.stream_of(gate))
    _capi.check(status, "fd_swiglu_out")
    _write_back(ly, out)


# ------------------------------------------------------------------ RoPE
def rope_out(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: torch.Tensor) -> None:
    """Rotate-half RoPE with cos/sin already broadcast (reference kernels.py:541-578)."""
    lx, lc, ls, ly = row_layout(x), row_layout(cos), row_layout(sin), row_layout(out)
    _same_grid(lx, lc, "cos")
    _same_grid(lx, ls, "sin")
    _same_grid(lx, ly, "out")
    if not _runnable(lx):
        return
    lib = _capi.load()
    status = lib.fd_rope_out(
        _capi.rows(lx), _capi.rows(lc), _capi.rows(ls), _capi.rows(ly), _capi.stream_of(x)
    )
    _capi.check(status, "fd_rope_out")
    _write_back(ly, out)


# ------------------------------------------------------------------ GEMV
def resolve_kind(kind: str | None) -> str:
    """``kind`` or ``$FUSED_DECODE_LINEAR_KIND`` (default "dot"); reference kernels.py:581-586."""
    if kind is None:
        kind = os.environ.get("FUSED_DECODE_LINEAR_KIND", "dot")
    if kind not in ("dot", "simt"):
        raise ValueError("kind must be 'dot' or 'simt'")
    return kind


def linear_config(kind: str, n: int, k: int) -> tuple[int, int, int, int]:
    """Default tile geometry of the GEMV: (block rows, columns per step, consumer warps, ring stages).

    Replaces the reference's hand tile table (kernels.py:589-603).  The
    stream-K kernel balances any (N, K) over the SMs, so one geometry serves
    every shape; ``FUSED_DECODE_LINEAR`` is accepted and ignored.
    """
    resolve_kind(kind)
    return GEMV_BLOCK_ROWS, GEMV_K_STEP, GEMV_WARPS, GEMV_STAGES


def linear_out(
    x: torch.Tensor,
    weight: torch.Tensor,
    y: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    row_add: torch.Tensor | None = None,
    kind: str | None = None,
) -> None:
    """``y = x @ weight.T [+ bias] [+ row_add]`` for ``x`` [M, K], M <= 16.

    Same contract as reference kernels.py:741-830: ``row_add`` is 2-D with
    each dim 1 or full (stride 0 where it broadcasts).
    """
    kind = resolve_kind(kind)
    m, k = x.shape
    n, k_w = weight.shape
    if k != k_w:
        raise ValueError(f"K mismatch: x has {k}, weight has {k_w}")
    if y.shape != (m, n):
        raise ValueError(f"y shape {tuple(y.shape)} != {(m, n)}")
    if m > GEMV_MAX_M:
        raise ValueError("linear_out only covers M <= 16")
    if m == 0 or n == 0:
        return
    lib = _capi.load()
    if bias is not None:
        bias_ptr, bias_dt, sbias = bias.data_ptr(), _capi.dtype_code(bias.dtype), int(bias.stride(0))
    else:
        bias_ptr, bias_dt, sbias = None, 0, 0
    if row_add is not None:
        ra_ptr, ra_dt = row_add.data_ptr(), _capi.dtype_code(row_add.dtype)
        srm = 0 if row_add.shape[0] == 1 else int(row_add.stride(0))
        srn = 0 if row_add.shape[1] == 1 else int(row_add.stride(1))
    else:
        ra_ptr, ra_dt, srm, srn = None, 0, 0, 0
    ws_bytes = lib.fd_linear_workspace_bytes(m, n, k)
    ws = WORKSPACES.get(x.device, ws_bytes)
    status = lib.fd_linear_out(
        x.data_ptr(), int(x.stride(0)), int(x.stride(1)),
        weight.data_ptr(), int(weight.stride(0)), int(weight.stride(1)),
        bias_ptr, bias_dt, sbias,
        ra_ptr, ra_dt, srm, srn,
        y.data_ptr(), int(y.stride(0)), int(y.stride(1)),
        _capi.dtype_code(x.dtype), m, n, k,
        _capi.FD_KIND_DOT if kind == "dot" else _capi.FD_KIND_SIMT,
        ws.data_ptr(), ws.numel(), _capi.stream_of(x),
    )
    _capi.check(status, "fd_linear_out")


# ------------------------------------------------------------------ fused MLP
def mlp_fusable(hidden2: torch.Tensor, norm_weight: torch.Tensor, w_gate_up: torch.Tensor,
                w_down: torch.Tensor) -> bool:
    """True when the two-kernel fused MLP can address these operands."""
    m, h = hidden2.shape
    i = w_down.shape[1]
    if not (1 <= m <= GEMV_MAX_M) or h % 8 or i % 8 or i == 0:
        return False
    if not hidden2.is_contiguous() or norm_weight.stride(0) != 1:
        return False
    if w_gate_up.stride(1) != 1 or w_down.stride(1) != 1:
        return False
    if w_gate_up.stride(0) % 8 or w_down.stride(0) % 8:
        return False
    for t in (hidden2, norm_weight, w_gate_up, w_down):
        if t.data_ptr() % 16:
            return False
    # Shared memory of the gate/up kernel with its smallest ring (2 stages of
    # 32 KB) in either mode: the RMSNorm'd batch (h padded to 128 columns)
    # and a copy of the norm weight, or the streamed normalised batch's 2 x 2
    # box slots (fd_stream.cuh: ring_smem_bytes, gateup_region_bytes,
    # linear_x_bytes).
    ks = -(-h // 128)
    nes = 4 if norm_weight.dtype == torch.float32 else 2
    fixed = 1024 + 2 * 32768 + 64 * 16 * 4 + 2 * 12 * 8
    resident = fixed + ks * 2 * m * 128 + ((h * nes + 15) & ~15)
    streamed = fixed + 2 * 2 * (1024 if m <= 8 else 2048)
    return min(resident, streamed) <= 227 * 1024 - 1024


def post_attn_mlp_out(
    hidden2: torch.Tensor,
    norm_weight: torch.Tensor,
    w_gate_up: torch.Tensor,
    w_down: torch.Tensor,
    out2: torch.Tensor,
    eps: float,
    kind: str,
    add_residual: bool = True,
) -> None:
    """Fused RMSNorm -> gate/up GEMV -> SwiGLU -> down GEMV (+ hidden) into ``out2``.

    Two kernel launches instead of the reference's four (ops.py:312-315).
    ``out2`` is [M, H] of the activation dtype, or float32 for the unrounded
    sum.  ``add_residual=False`` leaves out the residual, as a tensor-parallel
    rank does before its allreduce.
    """
    m, h = hidden2.shape
    i = w_down.shape[1]
    lib = _capi.load()
    ws_bytes = lib.fd_post_attn_mlp_workspace_bytes(m, h, i)
    ws = WORKSPACES.get(hidden2.device, ws_bytes)
    status = lib.fd_post_attn_mlp_out(
        hidden2.data_ptr(), norm_weight.data_ptr(), _capi.dtype_code(norm_weight.dtype),
        w_gate_up.data_ptr(), int(w_gate_up.stride(0)),
        w_down.data_ptr(), int(w_down.stride(0)),
        out2.data_ptr(), _capi.dtype_code(out2.dtype), _capi.dtype_code(hidden2.dtype), m, h, i,
        float(eps),
        _capi.FD_KIND_DOT if kind == "dot" else _capi.FD_KIND_SIMT,
        1 if add_residual else 0,
        ws.data_ptr(), ws.numel(), _capi.stream_of(hidden2),
    )
    _capi.check(status, "fd_post_attn_mlp_out")


def post_attn_mlp_stack_out(
    hidden2: torch.Tensor,
    layers,
    out2: torch.Tensor,
    eps: float,
    kind: str,
) -> None:
    """``len(layers)`` post_attn_mlp layers ``(norm_weight, w_gate_up, w_down)``
    enqueued by one library call (two launches per layer); the last output
    lands in ``out2``."""
    if not layers:
        raise ValueError("need at least one layer")
    m, h = hidden2.shape
    nw0, wgu0, wd0 = layers[0]
    i = wd0.shape[1]
    for nw, wgu, wd in layers:
        if (wgu.shape != wgu0.shape or wd.shape != wd0.shape or wgu.stride() != wgu0.stride()
                or wd.stride() != wd0.stride() or nw.dtype != nw0.dtype or nw.shape != nw0.shape):
            raise ValueError("all layers must share shapes, strides and dtypes")
    lib = _capi.load()
    ws = WORKSPACES.get(hidden2.device, lib.fd_post_attn_mlp_workspace_bytes(m, h, i))
    status = lib.fd_post_attn_mlp_stack_out(
        hidden2.data_ptr(), len(layers),
        _capi.ptr_array([nw.data_ptr() for nw, _, _ in layers]), _capi.dtype_code(nw0.dtype),
        _capi.ptr_array([wgu.data_ptr() for _, wgu, _ in layers]), int(wgu0.stride(0)),
        _capi.ptr_array([wd.data_ptr() for _, _, wd in layers]), int(wd0.stride(0)),
        out2.data_ptr(), _capi.dtype_code(hidden2.dtype), m, h, i, float(eps),
        _capi.FD_KIND_DOT if kind == "dot" else _capi.FD_KIND_SIMT,
        ws.data_ptr(), ws.numel(), _capi.stream_of(hidden2),
    )
    _capi.check(status, "fd_post_attn_mlp_stack_out")


def post_attn_mlp_tp_out(
    hidden2: torch.Tensor,
    norm_weight: torch.Tensor,
    w_gate_up_shard: torch.Tensor,
    w_down_shard: torch.Tensor,
    out2: torch.Tensor,
    eps: float,
    kind: str,
    exchange,
) -> None:
    """One tensor-parallel MLP layer whose allreduce runs over the NVLink
    exchange buffers of ``exchange`` (a ``fused_decode_b200.tp.TPExchange``):
    ``out2 = round(sum over ranks of the shard partials + hidden2)``."""
    m, h = hidden2.shape
    i = w_down_shard.shape[1]
    if m > exchange.m_max:
        raise ValueError(f"batch {m} exceeds the exchange's m_max={exchange.m_max}")
    if h != exchange.hidden:
        raise ValueError(f"hidden width {h} does not match the exchange's {exchange.hidden}")
    lib = _capi.load()
    ws = WORKSPACES.get(hidden2.device, lib.fd_post_attn_mlp_workspace_bytes(m, h, i))
    status = lib.fd_post_attn_mlp_tp_out(
        hidden2.data_ptr(), norm_weight.data_ptr(), _capi.dtype_code(norm_weight.dtype),
        w_gate_up_shard.data_ptr(), int(w_gate_up_shard.stride(0)),
        w_down_shard.data_ptr(), int(w_down_shard.stride(0)),
        out2.data_ptr(), _capi.dtype_code(hidden2.dtype), m, h, i, float(eps),
        _capi.FD_KIND_DOT if kind == "dot" else _capi.FD_KIND_SIMT,
        exchange.rank, exchange.world, exchange.pointers, exchange.m_max,
        ws.data_ptr(), ws.numel(), _capi.stream_of(hidden2),
    )
    _capi.check(status, "fd_post_attn_mlp_tp_out")


def post_attn_mlp_tp_stack_out(
    hidden2: torch.Tensor,
    layers,
    out2: torch.Tensor,
    eps: float,
    kind: str,
    exchange,
) -> None:
    """``len(layers)`` tensor-parallel MLP layers ``(norm_weight, w_gate_up
    shard, w_down shard)`` enqueued by one library call (three launches per
    layer, two under FD_TP_FOLD=1, or one persistent kernel per 32 layers
    under FD_STACK_PERSISTENT=1) whose partial sums travel through the NVLink
    exchange buffers of ``exchange``; the last output lands in ``out2`` on
    every rank."""
    if not layers:
        raise ValueError("need at least one layer")
    m, h = hidden2.shape
    nw0, wgu0, wd0 = layers[0]
    i = wd0.shape[1]
    if m > exchange.m_max:
        raise ValueError(f"batch {m} exceeds the exchange's m_max={exchange.m_max}")
    if h != exchange.hidden:
        raise ValueError(f"hidden width {h} does not match the exchange's {exchange.hidden}")
    for nw, wgu, wd in layers:
        if (wgu.shape != wgu0.shape or wd.shape != wd0.shape or wgu.stride() != wgu0.stride()
                or wd.stride() != wd0.stride() or nw.dtype != nw0.dtype or nw.shape != nw0.shape):
            raise ValueError("all layers must share shapes, strides and dtypes")
    lib = _capi.load()
    ws = WORKSPACES.get(hidden2.device, lib.fd_post_attn_mlp_workspace_bytes(m, h, i))
    status = lib.fd_post_attn_mlp_tp_stack_out(
        hidden2.data_ptr(), len(layers),
        _capi.ptr_array([nw.data_ptr() for nw, _, _ in layers]), _capi.dtype_code(nw0.dtype),
        _capi.ptr_array([wgu.data_ptr() for _, wgu, _ in layers]), int(wgu0.stride(0)),
        _capi.ptr_array([wd.data_ptr() for _, _, wd in layers]), int(wd0.stride(0)),
        out2.data_ptr(), _capi.dtype_code(hidden2.dtype), m, h, i, float(eps),
        _capi.FD_KIND_DOT if kind == "dot" else _capi.FD_KIND_SIMT,
        exchange.rank, exchange.world, exchange.pointers, exchange.m_max,
        ws.data_ptr(), ws.numel(), _capi.stream_of(hidden2),
    )
    _capi.check(status, "fd_post_attn_mlp_tp_stack_out")


def mlp_gate_up_out(
    hidden2: torch.Tensor,
    norm_weight: torch.Tensor,
    w_gate_up: torch.Tensor,
    mid: torch.Tensor,
    eps: float,
    kind: str,
) -> None:
    """First MLP kernel alone: ``mid = silu(gate) * up`` of the RMSNorm'd rows."""
    m, h = hidden2.shape
    i = mid.shape[1]
    lib = _capi.load()
    ws = WORKSPACES.get(hidden2.device, lib.fd_post_attn_mlp_workspace_bytes(m, h, i))
    status = lib.fd_mlp_gate_up_out(
        hidden2.data_ptr(), norm_weight.data_ptr(), _capi.dtype_code(norm_weight.dtype),
        w_gate_up.data_ptr(), int(w_gate_up.stride(0)), mid.data_ptr(),
        _capi.dtype_code(hidden2.dtype), m, h, i, float(eps),
        _capi.FD_KIND_DOT if kind == "dot" else _capi.FD_KIND_SIMT,
        ws.data_ptr(), ws.numel(), _capi.stream_of(hidden2),
    )
    _capi.check(status, "fd_mlp_gate_up_out")


def residual_add_out(partial: torch.Tensor, residual: torch.Tensor, out: torch.Tensor) -> None:
    """``out = round(partial + residual)``: fp32 partial sum + residual stream."""
    if partial.dtype != torch.float32 or not partial.is_contiguous():
        raise ValueError("partial must be a contiguous float32 tensor")
    if not residual.is_contiguous() or not out.is_contiguous():
        raise ValueError("residual and out must be contiguous")
    if partial.numel() != residual.numel() or out.numel() != residual.numel():
        raise ValueError("partial, residual and out must have the same number of elements")
    lib = _capi.load()
    status = lib.fd_residual_add_out(
        partial.data_ptr(), residual.data_ptr(), out.data_ptr(), _capi.dtype_code(out.dtype),
        out.numel(), _capi.stream_of(out),
    )
    _capi.check(status, "fd_residual_add_out")


# ------------------------------------------------------------------ roofs
def launch_copy(dst: torch.Tensor, src: torch.Tensor) -> None:
    """``dst[:] = src`` with the 16-byte streaming copy (reference kernels.py:849-852)."""
    nbytes = src.numel() * src.element_size()
    if dst.numel() * dst.element_size() < nbytes:
        raise ValueError("dst is smaller than src")
    lib = _capi.load()
    _capi.check(lib.fd_copy(dst.data_ptr(), src.data_ptr(), nbytes, _capi.stream_of(src)), "fd_copy")


def launch_triad(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, scale: float = 1.0) -> None:
    """``c = a + b * scale`` (reference kernels.py:855-858)."""
    lib = _capi.load()
    status = lib.fd_triad(
        a.data_ptr(), b.data_ptr(), c.data_ptr(), a.numel(), _capi.dtype_code(a.dtype),
        float(scale), _capi.stream_of(a),
    )
    _capi.check(status, "fd_triad")
