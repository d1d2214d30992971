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
def test_custom_ops_match_oracle_and_compile():
    """On the GPU every registered op runs the kernels: each of the six checked
    against the CPU oracle at atol = rtol = 1e-2, and bit-equal to the Python
    operator.  torch.compile traces a block of them without graph breaks."""
    import numpy as np

    import fused_decode_b200 as fd
    from oracle import fd_oracle as O

    g = torch.Generator(device="cuda").manual_seed(0)
    bf = torch.bfloat16

    def rn(*shape, scale=1.0, dtype=bf):
        return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dtype)

    def npf(t):
        return t.detach().float().cpu().numpy()

    def close(a, ref, what):
        torch.testing.assert_close(a.float().cpu(), torch.from_numpy(np.ascontiguousarray(ref)), rtol=1e-2,
                                   atol=1e-2, msg=lambda s: f"{what}: {s}")

    x, r = rn(4, 512), rn(4, 512)
    w = (1 + 0.1 * torch.randn(512, device="cuda", generator=g)).to(bf)
    wgu, wd = rn(2048, 512, scale=0.02), rn(512, 1024, scale=0.02)

    y = OPS.rms_norm(x, w, 1e-5)
    close(y, O.rms_norm(npf(x), npf(w), 1e-5, O.BF16), "rms_norm")
    assert torch.equal(y, fd.rms_norm(x, w, 1e-5))

    y, res = OPS.add_rms_norm(x, r, w, 1e-5)
    y_ref, r_ref = O.add_rms_norm(npf(x), npf(r), npf(w), 1e-5, O.BF16)
    close(y, y_ref, "add_rms_norm")
    close(res, r_ref, "add_rms_norm residual")

    q, cos, sin = rn(2, 3, 8, 128), rn(3, 1, 128), rn(3, 1, 128)
    y = OPS.rope(q, cos, sin)
    close(y, O.rope(npf(q), np.broadcast_to(npf(cos), q.shape), np.broadcast_to(npf(sin), q.shape), O.BF16), "rope")
    assert torch.equal(y, fd.rope(q, cos, sin))

    gt, up = rn(3, 1024), rn(3, 1024)
    y = OPS.swiglu(gt, up)
    close(y, O.swiglu(npf(gt), npf(up), O.BF16), "swiglu")

    xl, wl, bl, ra = rn(5, 512), rn(768, 512, scale=0.02), rn(768, scale=0.02), rn(5, 768)
    y = OPS.linear_decode(xl, wl, bl, ra, "dot")
    close(y, O.linear(npf(xl), npf(wl), npf(bl), npf(ra), O.BF16), "linear_decode")
    assert torch.equal(y, fd.linear_decode(xl, wl, bl, row_add=ra, kind="dot"))

    y = OPS.post_attn_mlp(x, w, wgu, wd, 1e-5, None)
    close(y, O.post_attn_mlp(npf(x), npf(w), npf(wgu), npf(wd), 1e-5, O.BF16), "post_attn_mlp")
    assert torch.equal(y, fd.post_attn_mlp(x, w, wgu, wd, 1e-5))

    def block(t):
        h = OPS.rms_norm(t, w, 1e-5)
        return OPS.post_attn_mlp(h, w, wgu, wd, 1e-5, "dot")

    compiled = torch.compile(block, fullgraph=True, backend="eager")
    assert torch.equal(compiled(x), block(x))
