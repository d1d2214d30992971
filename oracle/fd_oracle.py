"""CPU oracle for the decode-step path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's correctness formulation
(``src/fused_decode/reference.py`` of the fused-decode reference).  It exists
to CHECK the CUDA kernels: only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it.  The product path
(``fused_decode_b200``) never calls it and has no CPU fallback.

Pinned: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors that ``tests/golden/make_golden.py`` produced by running the
reference's own ``reference.py`` (PyTorch on CPU) on seeded inputs.

Conventions.  Arrays are float32 numpy arrays whose values are exactly
representable in the activation dtype (``"float16"`` or ``"bfloat16"``); every
function does its math in float32 and returns float32 arrays holding the
values rounded to the activation dtype, at the same points where the
reference rounds.
"""

from __future__ import annotations

import numpy as np

F16 = "float16"
BF16 = "bfloat16"


# ----------------------------------------------------------------- rounding
def round_bf16(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 -> float32, round-to-nearest-even (torch's ``.to(bfloat16)``)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def round_f16(a: np.ndarray) -> np.ndarray:
    """float32 -> float16 -> float32, round-to-nearest-even."""
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == F16:
        return round_f16(a)
    if dtype == BF16:
        return round_bf16(a)
    if dtype == "float32":
        return np.asarray(a, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype}")


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Raw bfloat16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 values already rounded to bfloat16 -> raw uint16 bit patterns."""
    return (round_bf16(a).view(np.uint32) >> 16).astype(np.uint16)


def _f32(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32)


def _rsqrt(v: np.ndarray) -> np.ndarray:
    return (np.float32(1.0) / np.sqrt(v, dtype=np.float32)).astype(np.float32)


# ----------------------------------------------------------------- operators
def rms_norm(x, weight, eps: float, dtype: str) -> np.ndarray:
    """``y = x * rsqrt(mean(x^2) + eps) * w`` in fp32, one rounding.

    Follows ``rms_norm_reference`` (reference.py:14-18).
    """
    xf = _f32(x)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    y = xf * _rsqrt(var + np.float32(eps)) * _f32(weight)
    return round_to(y, dtype)


def add_rms_norm(x, residual, weight, eps: float, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """``s = x + r`` (fp32); returns ``(round(norm(s) * w), round(s))``.

    Follows ``add_rms_norm_reference`` (reference.py:21-30): the norm sees the
    unrounded fp32 sum.
    """
    s = _f32(x) + _f32(residual)
    var = np.mean(s * s, axis=-1, keepdims=True, dtype=np.float32)
    y = s * _rsqrt(var + np.float32(eps)) * _f32(weight)
    return round_to(y, dtype), round_to(s, dtype)


def silu(g: np.ndarray) -> np.ndarray:
    """``g * sigmoid(g)`` with the overflow-free sigmoid (reference kernels.py:448-451)."""
    g = _f32(g)
    e = np.exp(-np.abs(g), dtype=np.float32)
    sig = np.where(g >= 0, np.float32(1.0) / (np.float32(1.0) + e), e / (np.float32(1.0) + e))
    return (g * sig.astype(np.float32)).astype(np.float32)


def swiglu(gate, up, dtype: str) -> np.ndarray:
    """``round(silu(gate) * up)`` in fp32 (reference.py:33-35)."""
    return round_to(silu(gate) * _f32(up), dtype)


def rope(x, cos, sin, dtype: str) -> np.ndarray:
    """Rotate-half RoPE, cos/sin broadcast right-aligned (reference.py:38-47).

    ``o[:h] = x1*c1 - x2*s1``, ``o[h:] = x2*c2 + x1*s2``; both halves of cos and
    sin are used (they are not assumed to repeat).
    """
    xf = _f32(x)
    c = np.broadcast_to(_f32(cos), xf.shape)
    s = np.broadcast_to(_f32(sin), xf.shape)
    h = xf.shape[-1] // 2
    x1, x2 = xf[..., :h], xf[..., h:]
    o = np.concatenate((x1 * c[..., :h] - x2 * s[..., :h], x2 * c[..., h:] + x1 * s[..., h:]), axis=-1)
    return round_to(o, dtype)


def linear(x, weight, bias=None, row_add=None, dtype: str = BF16) -> np.ndarray:
    """``round(x @ W^T + bias + row_add)`` in fp32 (reference.py:50-63)."""
    xf = _f32(x)
    y = xf @ _f32(weight).T
    if bias is not None:
        y = y + _f32(bias)
    if row_add is not None:
        y = y + _f32(row_add).reshape(y.shape)
    return round_to(y.astype(np.float32), dtype)


def post_attn_mlp(hidden, norm_weight, w_gate_up, w_down, eps: float, dtype: str,
                  add_residual: bool = True) -> np.ndarray:
    """RMSNorm -> gate/up -> SwiGLU -> down + hidden, rounding ``normed``,
    ``gate_up`` and ``mid`` to the activation dtype (reference.py:66-79).

    ``add_residual=False`` omits ``+ hidden`` (one tensor-parallel partial).
    """
    i = np.asarray(w_down).shape[1]
    h = rms_norm(hidden, norm_weight, eps, dtype)
    gu = linear(h, w_gate_up, dtype=dtype)
    mid = swiglu(gu[..., :i], gu[..., i:], dtype)
    return linear(mid, w_down, row_add=_f32(hidden) if add_residual else None, dtype=dtype)


def post_attn_mlp_partial_f32(hidden, norm_weight, w_gate_up_shard, w_down_shard, eps: float,
                              dtype: str) -> np.ndarray:
    """One tensor-parallel rank's down-projection partial, left in fp32.

    ``w_gate_up_shard`` is the rank's [2*I/T, H] restack of its gate rows and
    the matching up rows; ``w_down_shard`` is its [H, I/T] column slice.
    """
    i = np.asarray(w_down_shard).shape[1]
    h = rms_norm(hidden, norm_weight, eps, dtype)
    gu = linear(h, w_gate_up_shard, dtype=dtype)
    mid = swiglu(gu[..., :i], gu[..., i:], dtype)
    return (_f32(mid) @ _f32(w_down_shard).T).astype(np.float32)


# ----------------------------------------------------------------- helpers
def ulp_distance(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """Distance in units of the activation dtype's last place between two
    arrays of representable values (0 = bit-identical)."""
    a = _f32(a)
    b = _f32(b)
    if dtype == BF16:
        ia = (a.view(np.uint32) >> 16).astype(np.int64)
        ib = (b.view(np.uint32) >> 16).astype(np.int64)
        sign = 0x8000
    else:
        ia = a.astype(np.float16).view(np.uint16).astype(np.int64)
        ib = b.astype(np.float16).view(np.uint16).astype(np.int64)
        sign = 0x8000
    # map sign-magnitude to a monotone integer line
    ia = np.where(ia & sign, -(ia & (sign - 1)), ia)
    ib = np.where(ib & sign, -(ib & (sign - 1)), ib)
    return np.abs(ia - ib)
