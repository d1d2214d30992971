"""Public operators: the reference's ``fused_decode`` API, on sm_100a kernels.

Signatures, defaults, argument checks and exception types follow the
reference's ``src/fused_decode/ops.py`` so that callers (and the reference's
own tests) can switch by changing the import.  Inference only: nothing here
records a backward.

Divergence from the reference, on purpose: ``DECODE_LINEAR_MAX_M`` is 16, not
1.  The reference stops its default dispatcher at M=1 because on its laptop GPU
cuBLAS won from M=2 (ops.py:16-19); the B200 kernels here cover the whole
decode range M=1..16.  Above 16 rows (prefill) ``linear_decode`` passes through
to ``torch.nn.functional.linear`` exactly as the reference does.

Each operator first offers its arguments to the compiled dispatch module
(``_fastpath``, csrc/fd_fastpath.cpp), which launches the common case --
CUDA tensors of supported dtypes, at most four dimensions, no copies needed
-- without Python in between.  It declines everything else, argument errors
included, and the code below handles those with the same kernels.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from fused_decode_b200._capi import fast_or_none as _fast
from fused_decode_b200.kernels import (
    GEMV_MAX_M,
    linear_out,
    mlp_fusable,
    post_attn_mlp_out,
    resolve_kind,
    rms_out,
    rope_out,
    swiglu_out,
)

DECODE_LINEAR_MAX_M = GEMV_MAX_M
_ACTIVATION = (torch.float16, torch.bfloat16)
_NORM_WEIGHT = (torch.float16, torch.bfloat16, torch.float32)
_ANGLE = (torch.float16, torch.bfloat16, torch.float32)

__all__ = [
    "DECODE_LINEAR_MAX_M",
    "add_rms_norm",
    "linear_decode",
    "post_attn_mlp",
    "rms_norm",
    "rope",
    "swiglu",
]


# ---------------------------------------------------------------- checks
# Messages and exception types match reference ops.py:34-69.
def _check_activation(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype not in _ACTIVATION:
        raise TypeError(f"{name} must be float16 or bfloat16, got {t.dtype}")


def _check_same(t: torch.Tensor, like: torch.Tensor, name: str) -> None:
    if t.shape != like.shape:
        raise ValueError(f"{name} shape {tuple(t.shape)} != {tuple(like.shape)}")
    if t.dtype != like.dtype:
        raise TypeError(f"{name} dtype {t.dtype} != {like.dtype}")
    if t.device != like.device:
        raise ValueError(f"{name} is on {t.device}, expected {like.device}")


def _check_norm_weight(weight: torch.Tensor, x: torch.Tensor) -> None:
    if weight.device != x.device:
        raise ValueError(f"weight is on {weight.device}, expected {x.device}")
    if weight.dtype not in _NORM_WEIGHT:
        raise TypeError("weight must be float16, bfloat16, or float32")
    if weight.ndim != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError(f"weight must have shape ({x.shape[-1]},), got {tuple(weight.shape)}")


def _check_eps(eps: float) -> float:
    eps = float(eps)
    if not math.isfinite(eps) or eps < 0:
        raise ValueError("eps must be a finite value >= 0")
    return eps


def _fresh(like: torch.Tensor) -> torch.Tensor:
    return torch.empty(like.shape, device=like.device, dtype=like.dtype)


# ---------------------------------------------------------------- norms
def rms_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """RMSNorm over the last dimension; ``weight`` is ``(N,)`` (reference ops.py:72-88)."""
    fp = _fast()
    done = fp.rms_norm(x, weight, eps, out) if fp is not None else None
    if done is not None:
        return done
    _check_activation(x, "x")
    _check_norm_weight(weight, x)
    eps = _check_eps(eps)
    if out is None:
        out = _fresh(x)
    else:
        _check_same(out, x, "out")
    rms_out(x, weight, eps, out)
    return out


def add_rms_norm(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    out: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``residual_out = x + residual``, then RMSNorm of that sum.

    Pass ``residual_out=residual`` to update the residual stream in place.  The
    norm sees the float32 sum, not the rounded stored residual (reference
    ops.py:91-119).
    """
    fp = _fast()
    done = fp.add_rms_norm(x, residual, weight, eps, out, residual_out) if fp is not None else None
    if done is not None:
        return done
    _check_activation(x, "x")
    _check_activation(residual, "residual")
    _check_same(residual, x, "residual")
    _check_norm_weight(weight, x)
    eps = _check_eps(eps)
    if out is None:
        out = _fresh(x)
    else:
        _check_same(out, x, "out")
    if residual_out is None:
        residual_out = _fresh(x)
    else:
        _check_same(residual_out, x, "residual_out")
    rms_out(x, weight, eps, out, residual=residual, residual_out=residual_out)
    return out, residual_out


# ---------------------------------------------------------------- rope
def _broadcast_angles(src: torch.Tensor, like: torch.Tensor, name: str) -> torch.Tensor:
    """Right-aligned PyTorch broadcasting of cos/sin to ``like`` (reference ops.py:122-135)."""
    if src.device != like.device:
        raise ValueError(f"{name} is on {src.device}, expected {like.device}")
    if src.dtype not in _ANGLE:
        raise TypeError(f"{name} must be float16, bfloat16, or float32")
    if src.shape[-1] != like.shape[-1]:
        raise ValueError(f"{name} last dim {src.shape[-1]} != x last dim {like.shape[-1]}")
    try:
        return src.expand(like.shape)
    except RuntimeError as exc:
        raise ValueError(
            f"cannot broadcast {name} shape {tuple(src.shape)} to {tuple(like.shape)}"
        ) from exc


def rope(
    x: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Llama rotate-half RoPE on the last dimension (GPT-NeoX pairing).

    ``cos`` and ``sin`` broadcast over the leading dimensions (reference
    ops.py:138-160).
    """
    fp = _fast()
    done = fp.rope(x, cos, sin, out) if fp is not None else None
    if done is not None:
        return done
    _check_activation(x, "x")
    if x.shape[-1] % 2 != 0:
        raise ValueError("rope last dimension must be even")
    cos_b = _broadcast_angles(cos, x, "cos")
    sin_b = _broadcast_angles(sin, x, "sin")
    if out is None:
        out = _fresh(x)
    else:
        _check_same(out, x, "out")
    rope_out(x, cos_b, sin_b, out)
    return out


# ---------------------------------------------------------------- swiglu
def swiglu(
    gate: torch.Tensor,
    up: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``silu(gate) * up``: same shape, float32 math, stored in ``gate.dtype``."""
    fp = _fast()
    done = fp.swiglu(gate, up, out) if fp is not None else None
    if done is not None:
        return done
    _check_activation(gate, "gate")
    _check_activation(up, "up")
    _check_same(up, gate, "up")
    if out is None:
        out = _fresh(gate)
    else:
        _check_same(out, gate, "out")
    swiglu_out(gate, up, out)
    return out


# ---------------------------------------------------------------- linear
def _as_mk(x: torch.Tensor) -> tuple[torch.Tensor, tuple[int, ...] | None]:
    """View ``x`` as [M, K]; ``None`` leading dims marks a 1-D input (reference ops.py:181-192)."""
    k = x.shape[-1]
    if x.ndim == 1:
        return x.contiguous().view(1, k), None
    leading = tuple(x.shape[:-1])
    if x.ndim == 2 and min(x.stride()) >= 0:
        return x, leading
    return x.contiguous().view(-1, k), leading


def _as_row_add(row_add: torch.Tensor, m: int, n: int, expected: tuple[int, ...]) -> torch.Tensor:
    """``row_add`` as a 2-D [1|M, 1|N] operand (reference ops.py:195-209)."""
    if row_add.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("row_add must be float16, bfloat16, or float32")
    if row_add.ndim == 1 and row_add.numel() == n:
        return row_add.view(1, n)
    if row_add.shape == torch.Size(expected) and row_add.is_contiguous():
        return row_add.view(m, n)
    if row_add.ndim == 2 and row_add.shape[0] in (1, m) and row_add.shape[1] in (1, n):
        return row_add
    try:
        return row_add.expand(expected).contiguous().view(m, n)
    except RuntimeError as exc:
        raise ValueError(
            f"row_add shape {tuple(row_add.shape)} is not broadcastable to {expected}"
        ) from exc


def _torch_linear(x2, weight, bias, ra, dtype):
    produced = F.linear(x2, weight, bias)
    if ra is not None:
        produced = (produced.float() + ra.float()).to(dtype=dtype)
    return produced


def linear_decode(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    row_add: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    kind: str | None = None,
) -> torch.Tensor:
    """``y = x @ weight.T + bias``, with an optional epilogue add.

    ``weight`` is ``[N, K]`` as in ``F.linear``.  Flattened batches of up to
    16 rows run the stream-K GEMV; wider batches pass through to ``F.linear``
    (reference ops.py:212-280).
    """
    fp = _fast()
    done = fp.linear_decode(x, weight, bias, row_add, out, kind) if fp is not None else None
    if done is not None:
        return done
    _check_activation(x, "x")
    if weight.ndim != 2:
        raise ValueError(f"weight must have shape [N, K], got {tuple(weight.shape)}")
    if weight.device != x.device or weight.dtype != x.dtype:
        raise ValueError("weight device and dtype must match x")
    n, k = weight.shape
    if x.shape[-1] != k:
        raise ValueError(f"x last dim {x.shape[-1]} != weight K {k}")
    hand_limit = GEMV_MAX_M if kind is not None else DECODE_LINEAR_MAX_M
    kind = resolve_kind(kind)
    x2, leading = _as_mk(x)
    m = x2.shape[0]
    expected = (n,) if leading is None else (*leading, n)
    if bias is not None:
        if bias.ndim != 1 or bias.shape[0] != n:
            raise ValueError(f"bias must have shape ({n},), got {tuple(bias.shape)}")
        if bias.device != x.device:
            raise ValueError("bias must be on the same device as x")
        if bias.dtype not in (x.dtype, torch.float32):
            raise TypeError("bias must match x or be float32")
    ra = None
    if row_add is not None:
        if row_add.device != x.device:
            raise ValueError("row_add must be on the same device as x")
        ra = _as_row_add(row_add, m, n, expected)
    if m > hand_limit and out is None:
        produced = _torch_linear(x2, weight, bias, ra, x.dtype)
        return produced.view(n) if x.ndim == 1 else produced.view(expected)
    if out is None:
        y_full = torch.empty(expected, device=x.device, dtype=x.dtype)
    else:
        if tuple(out.shape) != expected or out.dtype != x.dtype or out.device != x.device:
            raise ValueError(f"out must be a contiguous {expected} tensor of dtype {x.dtype}")
        if not out.is_contiguous():
            raise ValueError("out must be contiguous")
        y_full = out
    y2 = y_full.view(m, n)
    if m == 0 or n == 0:
        return y_full
    if m > hand_limit:
        y2.copy_(_torch_linear(x2, weight, bias, ra, x.dtype))
        return y_full
    linear_out(x2, weight, y2, bias=bias, row_add=ra, kind=kind)
    return y_full


# ---------------------------------------------------------------- MLP block
def post_attn_mlp(
    hidden: torch.Tensor,
    norm_weight: torch.Tensor,
    w_gate_up: torch.Tensor,
    w_down: torch.Tensor,
    eps: float = 1e-6,
    *,
    kind: str | None = None,
) -> torch.Tensor:
    """Llama post-attention block, without the attention itself.

    ``hidden`` is ``[..., H]``, ``w_gate_up`` is ``[2I, H]`` (gate stacked
    above up), ``w_down`` is ``[H, I]``.  Returns ``down(swiglu(gate_up(
    rmsnorm(hidden)))) + hidden`` (reference ops.py:283-315).  Up to 16 rows
    run as two fused kernels (norm + gate/up GEMV + SwiGLU, then down GEMV +
    residual); other layouts run the four separate operators.
    """
    fp = _fast()
    done = fp.post_attn_mlp(hidden, norm_weight, w_gate_up, w_down, eps, kind) if fp is not None else None
    if done is not None:
        return done
    _check_activation(hidden, "hidden")
    if w_gate_up.ndim != 2 or w_down.ndim != 2:
        raise ValueError("w_gate_up and w_down must be rank-2")
    two_i, h = w_gate_up.shape
    h_down, i = w_down.shape
    if two_i != 2 * i or h != h_down or hidden.shape[-1] != h:
        raise ValueError(
            f"expected w_gate_up [2I, H] and w_down [H, I] with hidden [..., H], "
            f"got {tuple(w_gate_up.shape)}, {tuple(w_down.shape)}, {tuple(hidden.shape)}"
        )
    if w_gate_up.dtype != hidden.dtype or w_down.dtype != hidden.dtype:
        raise TypeError("MLP weights must match hidden dtype")
    if w_gate_up.device != hidden.device or w_down.device != hidden.device:
        raise ValueError("MLP weights must be on the same device as hidden")
    _check_norm_weight(norm_weight, hidden)
    eps = _check_eps(eps)
    kind_r = resolve_kind(kind)
    hidden2 = hidden.reshape(-1, h) if hidden.ndim != 2 else hidden
    m = hidden2.shape[0] if hidden.ndim > 0 else 0
    if hidden.ndim >= 1 and m > 0 and mlp_fusable(hidden2, norm_weight, w_gate_up, w_down):
        out = torch.empty(hidden.shape, device=hidden.device, dtype=hidden.dtype)
        post_attn_mlp_out(hidden2, norm_weight, w_gate_up, w_down, out.view(m, h), eps, kind_r)
        return out
    normed = rms_norm(hidden, norm_weight, eps=eps)
    gate_up = linear_decode(normed, w_gate_up, kind=kind)
    gate, up = gate_up.split(i, dim=-1)
    return linear_decode(swiglu(gate, up), w_down, row_add=hidden, kind=kind)
