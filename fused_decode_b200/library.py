"""The operators as ``torch.library`` custom ops (namespace ``fused_decode_b200``).

``torch.ops.fused_decode_b200.<op>`` calls the same kernels as the Python
functions in ``ops``; each op also has a fake (meta) implementation that only
describes its output, so ``torch.compile`` and other tracers see through the
op without a graph break and without running it.  The ops are functional:
fresh outputs, no ``out=`` / ``residual_out=`` aliasing (use the Python
functions for those).
"""

from __future__ import annotations

import torch

from fused_decode_b200 import ops

_NS = "fused_decode_b200"


def _fresh(shape, like: torch.Tensor) -> torch.Tensor:
    return torch.empty(shape, device=like.device, dtype=like.dtype)


@torch.library.custom_op(f"{_NS}::rms_norm", mutates_args=())
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return ops.rms_norm(x, weight, eps)


@rms_norm.register_fake
def _(x, weight, eps=1e-6):
    return _fresh(x.shape, x)


@torch.library.custom_op(f"{_NS}::add_rms_norm", mutates_args=())
def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                 eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.add_rms_norm(x, residual, weight, eps)


@add_rms_norm.register_fake
def _(x, residual, weight, eps=1e-6):
    return _fresh(x.shape, x), _fresh(x.shape, x)


@torch.library.custom_op(f"{_NS}::rope", mutates_args=())
def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return ops.rope(x, cos, sin)


@rope.register_fake
def _(x, cos, sin):
    return _fresh(x.shape, x)


@torch.library.custom_op(f"{_NS}::swiglu", mutates_args=())
def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return ops.swiglu(gate, up)


@swiglu.register_fake
def _(gate, up):
    return _fresh(gate.shape, gate)


@torch.library.custom_op(f"{_NS}::linear_decode", mutates_args=())
def linear_decode(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                  row_add: torch.Tensor | None = None, kind: str | None = None) -> torch.Tensor:
    return ops.linear_decode(x, weight, bias, row_add=row_add, kind=kind)


@linear_decode.register_fake
def _(x, weight, bias=None, row_add=None, kind=None):
    return _fresh((*x.shape[:-1], weight.shape[0]), x)


@torch.library.custom_op(f"{_NS}::post_attn_mlp", mutates_args=())
def post_attn_mlp(hidden: torch.Tensor, norm_weight: torch.Tensor, w_gate_up: torch.Tensor,
                  w_down: torch.Tensor, eps: float = 1e-6, kind: str | None = None) -> torch.Tensor:
    return ops.post_attn_mlp(hidden, norm_weight, w_gate_up, w_down, eps, kind=kind)


@post_attn_mlp.register_fake
def _(hidden, norm_weight, w_gate_up, w_down, eps=1e-6, kind=None):
    return _fresh(hidden.shape, hidden)
