"""A stack of post-attention MLP layers replayed as one CUDA graph.

The reference times ``post_attn_mlp`` inside a CUDA graph (bench.py:451-472)
to take host launch cost out of the step.  ``MlpStack`` is that as a reusable
object: it captures the whole stack on a private stream, and ``__call__``
copies the input into the graph's static buffer, replays, and returns the
static output.  By default the whole stack is enqueued by one library call
(``fd_post_attn_mlp_stack_out``: two programmatic-dependent launches per
layer, or one persistent kernel per 32 layers with FD_STACK_PERSISTENT=1;
intermediates in the library workspace).  With ``exchange=`` (a
``fused_decode_b200.tp.TPExchange``) the layers are this rank's
tensor-parallel shards and the call is ``fd_post_attn_mlp_tp_stack_out``
(three launches per layer, two with the rank sum in the down projection's
epilogue under FD_TP_FOLD=1, or one persistent kernel with the rank reduction
inside it under FD_STACK_PERSISTENT=1).  ``fused=False`` captures one
``post_attn_mlp`` call per layer instead, and ``layer_fn`` captures any per-layer callable (the
tensor-parallel layer of ``fused_decode_b200.tp``, for one).
"""

from __future__ import annotations

from typing import Sequence

import torch

from fused_decode_b200 import _capi
from fused_decode_b200 import kernels as K
from fused_decode_b200.ops import _check_activation, post_attn_mlp


class MlpStack:
    """``layers`` of ``(norm_weight, w_gate_up, w_down)`` applied in order.

    ``batch`` rows of width H are fixed at construction (a CUDA graph has
    static shapes).  Replays are stream-ordered on the caller's current
    stream.
    """

    def __init__(
        self,
        layers: Sequence[tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
        batch: int,
        eps: float = 1e-6,
        *,
        kind: str | None = None,
        layer_fn=None,
        fused: bool | None = None,
        exchange=None,
    ) -> None:
        if not layers:
            raise ValueError("need at least one layer")
        nw0, wgu0, wd0 = layers[0]
        _check_activation(wgu0, "w_gate_up")
        self.layers = list(layers)
        self.eps = float(eps)
        self.kind = K.resolve_kind(kind)
        self.h = int(wgu0.shape[1])
        self.device = wgu0.device
        self.dtype = wgu0.dtype
        self.exchange = exchange
        if layer_fn is None and exchange is not None:
            from fused_decode_b200 import tp

            def layer_fn_tp(x, nw, wgu, wd):
                return tp.TPPostAttnMlp(nw, wgu, wd, self.eps, kind=self.kind, exchange=exchange)(x)

            self._fn = layer_fn_tp
        else:
            self._fn = layer_fn or (lambda x, nw, wgu, wd: post_attn_mlp(x, nw, wgu, wd, self.eps, kind=self.kind))
        self.static_in = torch.zeros(batch, self.h, device=self.device, dtype=self.dtype)
        can_fuse = layer_fn is None and all(
            K.mlp_fusable(self.static_in, nw, wgu, wd) for nw, wgu, wd in self.layers)
        if fused and not can_fuse:
            raise ValueError("these layers cannot run as one fused stack")
        self.fused = can_fuse if fused is None else bool(fused)
        self._stream = torch.cuda.Stream(device=self.device)
        self.graph = torch.cuda.CUDAGraph()
        self._capture()

    def _run(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused:
            out = torch.empty_like(x)
            if self.exchange is not None:
                K.post_attn_mlp_tp_stack_out(x, self.layers, out, self.eps, self.kind, self.exchange)
            else:
                K.post_attn_mlp_stack_out(x, self.layers, out, self.eps, self.kind)
            return out
        for nw, wgu, wd in self.layers:
            x = self._fn(x, nw, wgu, wd)
        return x

    def _capture(self) -> None:
        cur = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            self._run(self.static_in)  # first call sizes the workspace outside capture
        cur.wait_stream(self._stream)
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(self.graph, stream=self._stream):
            self.static_out = self._run(self.static_in)

    @property
    def launches_per_replay(self) -> int:
        """Kernel launches of this library per replay: one persistent kernel
        per 32 layers where the stack entry point runs one, else the layer's
        launches (two; a third where the gate/up stage streams the normalised
        rows; another for the tensor-parallel rank sum) per layer."""
        nw0, wgu0, wd0 = self.layers[0]
        if not self.fused:
            per_layer = _capi.load().fd_post_attn_mlp_layer_launches(
                int(self.static_in.shape[0]), self.h, int(wd0.shape[1]), _capi.dtype_code(nw0.dtype),
                _capi.FD_KIND_DOT if self.kind == "dot" else _capi.FD_KIND_SIMT,
                1 if self.exchange is not None else 0)
            return int(per_layer) * len(self.layers)
        if self.exchange is not None:
            return int(_capi.load().fd_post_attn_mlp_tp_stack_launches(
                len(self.layers), _capi.dtype_code(nw0.dtype), int(self.static_in.shape[0]), self.h,
                int(wd0.shape[1]), _capi.FD_KIND_DOT if self.kind == "dot" else _capi.FD_KIND_SIMT))
        return int(_capi.load().fd_post_attn_mlp_stack_launches(
            len(self.layers), _capi.dtype_code(nw0.dtype), int(self.static_in.shape[0]), self.h,
            int(wd0.shape[1]), _capi.FD_KIND_DOT if self.kind == "dot" else _capi.FD_KIND_SIMT))

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.static_out

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        """Copy ``hidden`` (device or pinned host) in, replay, return the output."""
        self.static_in.copy_(hidden, non_blocking=True)
        self.graph.replay()
        return self.static_out
