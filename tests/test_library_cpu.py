"""The torch.library registrations: every op resolves under
torch.ops.fused_decode_b200 and its fake implementation gives the output the
real op returns (shape, dtype) for meta tensors -- no GPU, no kernel run."""

import pytest
import torch

import fused_decode_b200  # noqa: F401  (registers the ops)

OPS = torch.ops.fused_decode_b200


def _m(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, device="meta", dtype=dtype)


def test_ops_registered():
    for name in ("rms_norm", "add_rms_norm", "rope", "swiglu", "linear_decode", "post_attn_mlp"):
        assert hasattr(OPS, name), name


def test_fake_shapes():
    x = _m(3, 4096)
    assert OPS.rms_norm(x, _m(4096), 1e-5).shape == (3, 4096)
    y, r = OPS.add_rms_norm(x, _m(3, 4096), _m(4096, dtype=torch.float32), 1e-5)
    assert y.shape == r.shape == (3, 4096) and y.dtype == torch.bfloat16
    q = _m(1, 2048, 32, 128, dtype=torch.float16)
    assert OPS.rope(q, _m(2048, 1, 128, dtype=torch.float16), _m(2048, 1, 128, dtype=torch.float16)).shape == q.shape
    assert OPS.swiglu(_m(2, 14336), _m(2, 14336)).shape == (2, 14336)
    assert OPS.linear_decode(_m(8, 4096), _m(14336, 4096), None, None, None).shape == (8, 14336)
    assert OPS.linear_decode(_m(4096), _m(1024, 4096), None, None, "simt").shape == (1024,)
    assert OPS.linear_decode(_m(2, 5, 64), _m(32, 64), _m(32), _m(2, 5, 32), "dot").shape == (2, 5, 32)
    h = OPS.post_attn_mlp(_m(1, 4096), _m(4096), _m(28672, 4096), _m(4096, 14336), 1e-5, None)
    assert h.shape == (1, 4096) and h.dtype == torch.bfloat16


@pytest.mark.gpu
def test_custom_ops_match_python_ops_and_compile():
    """On the GPU the registered ops run the kernels (the same bits as the
    Python functions), and torch.compile traces them without graph breaks."""
    import fused_decode_b200 as fd

    torch.manual_seed(0)
    x = torch.randn(4, 512, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(512, device="cuda", dtype=torch.bfloat16)
    wgu = torch.randn(2048, 512, device="cuda", dtype=torch.bfloat16) * 0.02
    wd = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16) * 0.02
    assert torch.equal(OPS.rms_norm(x, w, 1e-5), fd.rms_norm(x, w, 1e-5))
    assert torch.equal(OPS.post_attn_mlp(x, w, wgu, wd, 1e-5, None), fd.post_attn_mlp(x, w, wgu, wd, 1e-5))

    def block(t):
        h = OPS.rms_norm(t, w, 1e-5)
        return OPS.post_attn_mlp(h, w, wgu, wd, 1e-5, "dot")

    compiled = torch.compile(block, fullgraph=True, backend="eager")
    assert torch.equal(compiled(x), block(x))
