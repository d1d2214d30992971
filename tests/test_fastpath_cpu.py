"""The compiled dispatch module (``_fastpath``) on CPU: it loads next to the
library, exposes one function per operator plus the workspace cache, and
declines (returns None for) anything that is not a CUDA tensor, so argument
errors reach the Python checks and their reference messages."""

import pytest
import torch

from fused_decode_b200 import _capi

OPS = ("rms_norm", "add_rms_norm", "rope", "swiglu", "linear_decode", "post_attn_mlp")


@pytest.fixture(scope="module")
def fp():
    return _capi.fast()


def test_exports(fp):
    for name in OPS + ("workspace", "workspaces", "clear_workspaces"):
        assert callable(getattr(fp, name)), name
    assert _capi.fast_or_none() is fp


def test_declines_cpu_and_non_tensors(fp):
    x = torch.randn(2, 8, dtype=torch.float16)
    w = torch.ones(8, dtype=torch.float16)
    assert fp.rms_norm(x, w, 1e-6, None) is None
    assert fp.rms_norm([1.0], w, 1e-6, None) is None
    assert fp.add_rms_norm(x, x, w, 1e-6, None, None) is None
    assert fp.rope(x, x, x, None) is None
    assert fp.swiglu(x, x, None) is None
    assert fp.linear_decode(x, torch.ones(3, 8, dtype=torch.float16), None, None, None, None) is None
    assert fp.post_attn_mlp(x, w, torch.ones(32, 8, dtype=torch.float16),
                            torch.ones(8, 16, dtype=torch.float16), 1e-6, None) is None
    assert fp.workspaces() == []


@pytest.mark.parametrize("call", [
    lambda fd: fd.rms_norm(torch.randn(2, 8), torch.ones(8)),
    lambda fd: fd.swiglu(torch.randn(2, 8, dtype=torch.float16), torch.randn(2, 8, dtype=torch.float16)),
    lambda fd: fd.linear_decode(torch.randn(2, 8, dtype=torch.float16), torch.ones(3, 8, dtype=torch.float16)),
])
def test_errors_keep_reference_messages(call):
    import fused_decode_b200 as fd

    with pytest.raises((ValueError, TypeError), match="must be"):
        call(fd)
