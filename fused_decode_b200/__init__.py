"""B200-native (sm_100a) kernels for the non-attention half of a Llama decode step.

Drop-in for the reference package ``fused_decode``: the same operators, with
the same signatures and error behaviour, backed by hand-written CUDA kernels in
``libfd_b200.so`` (C ABI: ``include/fd_b200.h``).  ``import fused_decode_b200
as fused_decode`` is the switch.
"""

from fused_decode_b200.ops import (
    DECODE_LINEAR_MAX_M,
    add_rms_norm,
    linear_decode,
    post_attn_mlp,
    rms_norm,
    rope,
    swiglu,
)

__all__ = [
    "DECODE_LINEAR_MAX_M",
    "add_rms_norm",
    "linear_decode",
    "post_attn_mlp",
    "rms_norm",
    "rope",
    "swiglu",
]
__version__ = "0.1.0"

# torch.ops.fused_decode_b200.* (custom ops with fake implementations)
from fused_decode_b200 import library  # noqa: E402,F401
