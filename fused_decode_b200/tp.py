"""Tensor-parallel post-attention MLP (Megatron split) over NVLink.

Each of T ranks holds the gate rows ``[r*I/T, (r+1)*I/T)`` of ``w_gate_up``
together with the matching up rows ``I + [r*I/T, (r+1)*I/T)``, restacked as its
own ``[2I/T, H]`` weight, and the column slice ``w_down[:, r*I/T:(r+1)*I/T]``.
A layer is: the fused MLP kernels on the local shard with an fp32 partial and
no residual, a sum of the ``[M, H]`` fp32 partials over all ranks, then
``out = round(sum + hidden)``.  RMSNorm is recomputed on every rank (hidden is
replicated), so the sum is the only exchange.

Two ways to do the sum.  With a ``TPExchange`` (the default on GPUs), the
down-projection kernel itself stores its block partials into every rank's
exchange buffer over NVLink and a small kernel adds them up: three launches
per layer, no NCCL call, CUDA-graph capturable.  ``FD_TP_FOLD=1`` in the
environment moves that sum into the down projection's epilogue (the CTA that
finished a block waits for the other ranks' words of it): two launches per
layer, the same bits, and measured no faster on 2 and 4 B200s.  Without one, ``all_reduce``
over the process group (NCCL) and a residual-add launch.

The reference has no multi-GPU path; this is the tensor-parallel layout of
its ``post_attn_mlp`` (ops.py:283-315) that the B200 build adds.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from fused_decode_b200 import _capi
from fused_decode_b200 import kernels as K


def shard_bounds(inner: int, rank: int, world: int) -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if inner % world:
        raise ValueError(f"intermediate size {inner} is not divisible by {world} ranks")
    per = inner // world
    return rank * per, (rank + 1) * per


def shard_gate_up(w_gate_up: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's ``[2I/T, H]`` restack: its gate rows, then the matching up rows."""
    two_i = w_gate_up.shape[0]
    if two_i % 2:
        raise ValueError("w_gate_up must have an even number of rows [2I, H]")
    inner = two_i // 2
    lo, hi = shard_bounds(inner, rank, world)
    return torch.cat((w_gate_up[lo:hi], w_gate_up[inner + lo:inner + hi]), dim=0).contiguous()


def shard_down(w_down: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's ``[H, I/T]`` column slice of ``w_down`` (made contiguous)."""
    lo, hi = shard_bounds(w_down.shape[1], rank, world)
    return w_down[:, lo:hi].contiguous()


class TPExchange:
    """The NVLink exchange buffers of one tensor-parallel group.

    Every rank allocates one buffer (``fd_tp_exchange_alloc``) and maps every
    other rank's through CUDA IPC; the handles travel through the process
    group.  Collective: every rank constructs it, with the same ``hidden``
    and ``m_max``.  ``close()`` (also collective) unmaps and frees.
    """

    HANDLE_BYTES = 64

    def __init__(self, hidden: int, m_max: int = 16, group=None) -> None:
        self.group = group
        self.hidden = int(hidden)
        self.m_max = int(m_max)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        lib = _capi.load()
        buf = ctypes.c_void_p()
        _capi.check(lib.fd_tp_exchange_alloc(self.world, self.m_max, self.hidden, ctypes.byref(buf)),
                    "fd_tp_exchange_alloc")
        self._buf = buf.value
        self._peers: list[int] = []
        handle = ctypes.create_string_buffer(self.HANDLE_BYTES)
        _capi.check(lib.fd_tp_exchange_handle(self._buf, handle), "fd_tp_exchange_handle")
        handles = [handle.raw]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._buf)
                continue
            peer = ctypes.c_void_p()
            _capi.check(lib.fd_tp_exchange_open(ctypes.create_string_buffer(h, self.HANDLE_BYTES),
                                                ctypes.byref(peer)), "fd_tp_exchange_open")
            self._peers.append(peer.value)
            ptrs.append(peer.value)
        self.pointers = _capi.ptr_array(ptrs)
        if self.world > 1:
            dist.barrier(group=group)  # every rank has mapped every buffer

    def close(self) -> None:
        if self._buf is None:
            return
        lib = _capi.load()
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank still writes into a buffer
        for p in self._peers:
            lib.fd_tp_exchange_close(p)
        self._peers = []
        lib.fd_tp_exchange_free(self._buf)
        self._buf = None


class TPPostAttnMlp:
    """One tensor-parallel MLP layer on this rank.

    ``__call__(hidden)`` returns ``post_attn_mlp(hidden, ...)`` of the full
    (unsharded) weights on every rank.  All ranks must call it in the same
    order with the same ``hidden``.
    """

    def __init__(self, norm_weight, w_gate_up_shard, w_down_shard, eps=1e-6, *, kind=None,
                 group=None, exchange: TPExchange | None = None) -> None:
        self.norm_weight = norm_weight
        self.w_gate_up = w_gate_up_shard
        self.w_down = w_down_shard
        self.eps = float(eps)
        self.kind = K.resolve_kind(kind)
        self.group = group
        self.exchange = exchange
        if self.w_gate_up.shape[0] != 2 * self.w_down.shape[1]:
            raise ValueError("gate/up shard rows must be twice the down shard columns")
        if self.w_gate_up.shape[1] != self.w_down.shape[0]:
            raise ValueError("gate/up shard and down shard disagree on H")

    @classmethod
    def from_full(cls, norm_weight, w_gate_up, w_down, rank, world, eps=1e-6, *, kind=None, group=None,
                  exchange: TPExchange | None = None):
        return cls(norm_weight, shard_gate_up(w_gate_up, rank, world), shard_down(w_down, rank, world),
                   eps, kind=kind, group=group, exchange=exchange)

    def partial(self, hidden2: torch.Tensor) -> torch.Tensor:
        """This rank's fp32 ``[M, H]`` down-projection partial (no residual)."""
        m, h = hidden2.shape
        part = torch.empty(m, h, device=hidden2.device, dtype=torch.float32)
        K.post_attn_mlp_out(hidden2, self.norm_weight, self.w_gate_up, self.w_down, part, self.eps,
                            self.kind, add_residual=False)
        return part

    def finish(self, total: torch.Tensor, hidden2: torch.Tensor) -> torch.Tensor:
        """``round(total + hidden)``: the allreduced fp32 sum plus the residual."""
        out = torch.empty(hidden2.shape, device=hidden2.device, dtype=hidden2.dtype)
        K.residual_add_out(total, hidden2, out)
        return out

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        h = hidden.shape[-1]
        if self.w_gate_up.shape[1] != h:
            raise ValueError(f"hidden width {h} does not match the weights' H={self.w_gate_up.shape[1]}")
        hidden2 = hidden.reshape(-1, h).contiguous()
        if self.exchange is not None:
            out = torch.empty(hidden2.shape, device=hidden2.device, dtype=hidden2.dtype)
            K.post_attn_mlp_tp_out(hidden2, self.norm_weight, self.w_gate_up, self.w_down, out, self.eps,
                                   self.kind, self.exchange)
            return out.view(hidden.shape)
        part = self.partial(hidden2)
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        return self.finish(part, hidden2).view(hidden.shape)
