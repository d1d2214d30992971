"""The compiled dispatch (``_fastpath``) against the Python launchers on the
GPU: for every operator and several layouts, the fast path is taken (returns
a result, not None) and its output is bit-identical to the same kernels
launched through ``kernels.*_out``; layouts it must decline (five dims,
copies) return None.  Parity of both paths with the oracle is covered by the
operator tests, which now run through the fast path."""

import pytest
import torch

import fused_decode_b200 as fd
from fused_decode_b200 import _capi
from fused_decode_b200 import kernels as K

pytestmark = pytest.mark.gpu

F16, BF16 = torch.float16, torch.bfloat16


@pytest.fixture(scope="module")
def fp():
    return _capi.fast()


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("shape", [(1, 4096), (7, 3072), (2, 3, 100), (2, 2, 2, 64), (4096,)])
@pytest.mark.parametrize("wdt", ["same", torch.float32])
def test_norms(fp, dtype, shape, wdt):
    g = _gen(1)
    x = torch.randn(shape, device="cuda", dtype=dtype, generator=g)
    r = torch.randn(shape, device="cuda", dtype=dtype, generator=g)
    w = torch.randn(shape[-1], device="cuda", dtype=dtype if wdt == "same" else wdt, generator=g)
    y = fp.rms_norm(x, w, 1e-5, None)
    assert y is not None
    ref = torch.empty_like(x)
    K.rms_out(x, w, 1e-5, ref)
    assert torch.equal(y, ref)
    pair = fp.add_rms_norm(x, r, w, 1e-5, None, None)
    assert pair is not None
    ry, rro = torch.empty_like(x), torch.empty_like(x)
    K.rms_out(x, w, 1e-5, ry, residual=r, residual_out=rro)
    assert torch.equal(pair[0], ry) and torch.equal(pair[1], rro)


def test_add_rms_norm_in_place_residual(fp):
    g = _gen(2)
    x = torch.randn(4, 4096, device="cuda", dtype=BF16, generator=g)
    r = torch.randn(4, 4096, device="cuda", dtype=BF16, generator=g)
    w = torch.randn(4096, device="cuda", dtype=BF16, generator=g)
    want_y, want_r = torch.empty_like(x), torch.empty_like(x)
    K.rms_out(x, w, 1e-6, want_y, residual=r, residual_out=want_r)
    out = torch.empty_like(x)
    y, ro = fd.add_rms_norm(x, r, w, 1e-6, out=out, residual_out=r)
    assert y is out and ro is r
    assert torch.equal(out, want_y) and torch.equal(r, want_r)


def test_strided_views_and_declines(fp):
    g = _gen(3)
    base = torch.randn(8, 2 * 256, device="cuda", dtype=F16, generator=g)
    gate, up = base.split(256, dim=-1)  # strided views, as SwiGLU callers pass them
    y = fp.swiglu(gate, up, None)
    assert y is not None
    ref = torch.empty(8, 256, device="cuda", dtype=F16)
    K.swiglu_out(gate, up, ref)
    assert torch.equal(y, ref)
    five = torch.randn(2, 2, 2, 2, 64, device="cuda", dtype=F16, generator=g)
    assert fp.rms_norm(five, torch.ones(64, device="cuda", dtype=F16), 1e-6, None) is None
    assert fp.swiglu(five, five, None) is None
    # declined calls still compute, through the Python path
    assert torch.equal(fd.swiglu(five, five), fd.swiglu(five.reshape(-1, 64), five.reshape(-1, 64)).view(five.shape))


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("xs,cs", [((1, 1, 32, 128), (1, 1, 128)), ((1, 16, 8, 128), (16, 1, 128)),
                                   ((3, 64), (64,))])
def test_rope(fp, dtype, xs, cs):
    g = _gen(4)
    x = torch.randn(xs, device="cuda", dtype=dtype, generator=g)
    cos = torch.randn(cs, device="cuda", dtype=torch.float32, generator=g)
    sin = torch.randn(cs, device="cuda", dtype=torch.float32, generator=g)
    y = fp.rope(x, cos, sin, None)
    assert y is not None
    ref = torch.empty_like(x)
    K.rope_out(x, cos.expand(xs), sin.expand(xs), ref)
    assert torch.equal(y, ref)


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (3, 1000, 2048), (16, 512, 4096)])
@pytest.mark.parametrize("kind", ["dot", "simt"])
@pytest.mark.parametrize("extras", ["none", "bias", "bias32_row", "row1d"])
def test_linear(fp, dtype, m, n, k, kind, extras):
    g = _gen(5)
    x = torch.randn(m, k, device="cuda", dtype=dtype, generator=g) * k**-0.5
    w = torch.randn(n, k, device="cuda", dtype=dtype, generator=g) * k**-0.5
    bias = row = None
    if extras == "bias":
        bias = torch.randn(n, device="cuda", dtype=dtype, generator=g)
    elif extras == "bias32_row":
        bias = torch.randn(n, device="cuda", dtype=torch.float32, generator=g)
        row = torch.randn(m, n, device="cuda", dtype=dtype, generator=g)
    elif extras == "row1d":
        row = torch.randn(n, device="cuda", dtype=torch.float32, generator=g)
    y = fp.linear_decode(x, w, bias, row, None, kind)
    assert y is not None
    ref = torch.empty(m, n, device="cuda", dtype=dtype)
    ra = None if row is None else (row.view(1, n) if row.ndim == 1 else row)
    K.linear_out(x, w, ref, bias=bias, row_add=ra, kind=kind)
    assert torch.equal(y, ref)


def test_linear_shapes_and_declines(fp):
    g = _gen(6)
    w = torch.randn(256, 512, device="cuda", dtype=F16, generator=g)
    x1 = torch.randn(512, device="cuda", dtype=F16, generator=g)
    y1 = fp.linear_decode(x1, w, None, None, None, None)
    assert y1 is not None and y1.shape == (256,)
    assert torch.equal(y1, fd.linear_decode(x1.view(1, 512), w).view(256))
    x3 = torch.randn(2, 3, 512, device="cuda", dtype=F16, generator=g)
    y3 = fp.linear_decode(x3, w, None, None, None, None)
    assert y3 is not None and y3.shape == (2, 3, 256)
    ref = torch.empty(6, 256, device="cuda", dtype=F16)
    K.linear_out(x3.view(6, 512), w, ref)
    assert torch.equal(y3.view(6, 256), ref)
    out = torch.empty(2, 3, 256, device="cuda", dtype=F16)
    assert fp.linear_decode(x3, w, None, None, out, "dot") is out
    assert torch.equal(out, y3)
    x17 = torch.randn(17, 512, device="cuda", dtype=F16, generator=g)
    assert torch.equal(fp.linear_decode(x17, w, None, None, None, None), torch.nn.functional.linear(x17, w))
    assert fp.linear_decode(x3, w, None, None, None, "wide") is None
    with pytest.raises(ValueError, match="kind must be"):
        fd.linear_decode(x3, w, kind="wide")


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("m", [1, 8])
@pytest.mark.parametrize("kind", [None, "simt"])
def test_post_attn_mlp(fp, dtype, m, kind):
    g = _gen(7)
    h, i = 1024, 2816
    hid = torch.randn(m, h, device="cuda", dtype=dtype, generator=g)
    nw = torch.randn(h, device="cuda", dtype=dtype, generator=g)
    wgu = torch.randn(2 * i, h, device="cuda", dtype=dtype, generator=g) * h**-0.5
    wd = torch.randn(h, i, device="cuda", dtype=dtype, generator=g) * i**-0.5
    y = fp.post_attn_mlp(hid, nw, wgu, wd, 1e-5, kind)
    assert y is not None
    ref = torch.empty_like(hid)
    K.post_attn_mlp_out(hid, nw, wgu, wd, ref, 1e-5, K.resolve_kind(kind))
    assert torch.equal(y, ref)
    assert fp.post_attn_mlp(hid.t().contiguous().t(), nw, wgu, wd, 1e-5, kind) is None or m == 1


def test_workspaces_shared_and_clean(fp):
    x = torch.randn(4, 4096, device="cuda", dtype=BF16)
    w = torch.randn(4096, 4096, device="cuda", dtype=BF16)
    fd.linear_decode(x, w)
    torch.cuda.synchronize()
    keys = [k for k, _ in fp.workspaces()]
    assert keys and all(k[0] == torch.cuda.current_device() for k in keys)
    assert K.WORKSPACES.get(x.device, 1024).data_ptr() in {t.data_ptr() for _, t in fp.workspaces()}
    assert all(v == 0 for v in K.WORKSPACES.status().values())


def test_linear_wide_batch_passes_through(fp):
    g = _gen(8)
    x = torch.randn(4, 8, 512, device="cuda", dtype=BF16, generator=g)
    w = torch.randn(256, 512, device="cuda", dtype=BF16, generator=g)
    b = torch.randn(256, device="cuda", dtype=BF16, generator=g)
    y = fp.linear_decode(x, w, b, None, None, None)
    assert y is not None and y.shape == (4, 8, 256)
    assert torch.equal(y, torch.nn.functional.linear(x.view(32, 512), w, b).view(4, 8, 256))
    # forms the pass-through leaves to the Python path
    assert fp.linear_decode(x, w, b.float(), None, None, None) is None
    assert fp.linear_decode(x, w, None, torch.zeros(256, device="cuda", dtype=BF16), None, None) is None


def test_parameters_subclasses_and_modes(fp):
    g = _gen(9)
    x = torch.randn(3, 256, device="cuda", dtype=F16, generator=g)
    w = torch.nn.Parameter(torch.randn(256, device="cuda", dtype=F16, generator=g), requires_grad=False)
    y = fp.rms_norm(x, w, 1e-6, None)  # model weights are Parameters: fast path
    assert y is not None

    class Tagged(torch.Tensor):
        pass

    assert fp.rms_norm(x.as_subclass(Tagged), w, 1e-6, None) is None
    assert torch.equal(fd.rms_norm(x.as_subclass(Tagged), w).as_subclass(torch.Tensor), y)
    with torch.device("cuda"):  # a torch-function mode: declined, computed by the Python path
        assert fp.rms_norm(x, w, 1e-6, None) is None
        assert torch.equal(fd.rms_norm(x, w), y)
