"""PyTorch-eager CPU formulation of the decode MLP -- TEST AND BASELINE INFRASTRUCTURE ONLY.

The reference checks its kernels against a PyTorch formulation that runs
eagerly on the CPU (``src/fused_decode/reference.py:14-79``: fp32 math with
the activation dtype's rounding at fixed points, the GEMVs as fp32
``F.linear`` on the CPU).  This module restates that formulation for the one
place that needs it as a *timed* CPU path: the CPU baseline and the reference
arm of ``bench.py``, which time the reference's PyTorch-eager CPU path on the
host cores.  Tests pin it to the reference's golden vectors
(``tests/test_oracle_golden.py``).  The product path never imports it.

Tensors are CPU tensors in the activation dtype (bf16 or fp16); every
function returns tensors in that dtype.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """round(x * rsqrt(mean(x^2) + eps) * w), fp32 inside (reference.py:14-18)."""
    xf = x.float()
    scale = torch.rsqrt(xf.mul(xf).mean(dim=-1, keepdim=True).add(eps))
    return (xf * scale * weight.float()).to(x.dtype)


def linear(x: torch.Tensor, weight: torch.Tensor, row_add: torch.Tensor | None = None) -> torch.Tensor:
    """round(x @ W^T (+ row_add)) with an fp32 product on the CPU (reference.py:50-63)."""
    y = F.linear(x.float(), weight.float())
    if row_add is not None:
        y = y + row_add.float()
    return y.to(x.dtype)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """round(silu(gate) * up), fp32 inside (reference.py:33-35)."""
    return (F.silu(gate.float()) * up.float()).to(gate.dtype)


def post_attn_mlp(hidden: torch.Tensor, norm_weight: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                  eps: float) -> torch.Tensor:
    """The MLP block with the reference's three rounding points (reference.py:66-79):
    normed, gate_up and mid are rounded to the activation dtype; the residual
    is added in fp32 before the final rounding.  The weights are widened to
    fp32 on every call, as the reference's CPU path does."""
    i = w_down.shape[1]
    normed = rms_norm(hidden, norm_weight, eps)
    gate_up = linear(normed, w_gate_up)
    mid = swiglu(gate_up[..., :i], gate_up[..., i:])
    return linear(mid, w_down, row_add=hidden)
