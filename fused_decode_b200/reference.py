"""PyTorch fp32 references of the operators, for correctness checks.

The same module and function names as the reference package's
``fused_decode.reference`` (src/fused_decode/reference.py:14-79), so callers'
tests that compare against it keep working after the import switch.  No
operator in this package calls these; they are the yardstick, not a fallback.

Every reference computes in fp32 and rounds once to the activation dtype at
the point where the kernels round: the norms and SwiGLU round their output,
``post_attn_mlp_reference`` rounds the normed row, the gate/up product and the
SwiGLU output before the down projection (the reference's three rounding
points, reference.py:66-79).  The GEMV references run on the CPU so that no
TF32 tensor-core path can narrow the fp32 product.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

__all__ = [
    "add_rms_norm_reference",
    "linear_reference",
    "post_attn_mlp_reference",
    "rms_norm_reference",
    "rope_reference",
    "swiglu_reference",
]


def _normalize(s: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    inv = torch.rsqrt(s.square().mean(dim=-1, keepdim=True) + eps)
    return s * inv * weight.float()


def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``x * rsqrt(mean(x^2) + eps) * weight`` (reference.py:14-18)."""
    return _normalize(x.float(), weight, eps).to(x.dtype)


def add_rms_norm_reference(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6
) -> tuple[torch.Tensor, torch.Tensor]:
    """``(norm(x + residual), x + residual)``; the norm sees the unrounded
    fp32 sum (reference.py:21-30)."""
    s = x.float() + residual.float()
    return _normalize(s, weight, eps).to(x.dtype), s.to(x.dtype)


def swiglu_reference(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` in fp32 (reference.py:33-35)."""
    return (F.silu(gate.float()) * up.float()).to(gate.dtype)


def rope_reference(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE with cos/sin broadcast to x (reference.py:38-47):
    ``[x1 c1 - x2 s1, x2 c2 + x1 s2]`` over the two halves of the last dim."""
    xf = x.float()
    c = cos.float().expand(x.shape)
    s = sin.float().expand(x.shape)
    x1, x2 = xf.chunk(2, dim=-1)
    c1, c2 = c.chunk(2, dim=-1)
    s1, s2 = s.chunk(2, dim=-1)
    return torch.cat((x1 * c1 - x2 * s1, x2 * c2 + x1 * s2), dim=-1).to(x.dtype)


def linear_reference(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    row_add: torch.Tensor | None = None,
) -> torch.Tensor:
    """``x @ weight.T (+ bias) (+ row_add)`` in fp32 on the CPU, one rounding
    at the end, returned on x's device (reference.py:50-63)."""
    cpu = lambda t: t.detach().float().cpu()  # noqa: E731
    y = F.linear(cpu(x), cpu(weight), None if bias is None else cpu(bias))
    if row_add is not None:
        y = y + cpu(row_add).reshape(y.shape)
    return y.to(device=x.device, dtype=x.dtype)


def post_attn_mlp_reference(
    hidden: torch.Tensor,
    norm_weight: torch.Tensor,
    w_gate_up: torch.Tensor,
    w_down: torch.Tensor,
    eps: float = 1e-6,
) -> torch.Tensor:
    """``down(swiglu(split(gate_up(rmsnorm(hidden))))) + hidden``, rounded at
    the same three points as the kernels (reference.py:66-79)."""
    i = w_down.shape[1]
    normed = rms_norm_reference(hidden, norm_weight, eps)
    gate_up = linear_reference(normed, w_gate_up)
    mid = swiglu_reference(gate_up[..., :i], gate_up[..., i:])
    return linear_reference(mid, w_down, row_add=hidden)
