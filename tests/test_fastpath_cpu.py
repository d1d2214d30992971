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


# ---- the arguments the fast path derives, against the Python path's --------
from fused_decode_b200 import kernels as K  # noqa: E402
from fused_decode_b200 import ops as O  # noqa: E402


def _layouts():
    g = torch.Generator().manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    base = r(6, 10, 12)
    yield "contig2d", r(5, 64)
    yield "contig1d", r(64)
    yield "strided1d", r(128)[::2]
    yield "contig3d", base
    yield "contig4d", r(2, 3, 4, 16)
    yield "transposed", r(64, 5).t()
    yield "col_slice", base[:, :, :8]
    yield "row_slice", base[1:5, ::3]
    yield "permuted", base.permute(1, 0, 2)
    yield "expanded", r(1, 12).expand(7, 12)
    yield "expanded3d", r(1, 1, 12).expand(2, 3, 12)
    yield "split_view", r(4, 32).split(16, dim=-1)[1]
    yield "five_dims", r(2, 2, 2, 2, 8)
    yield "empty", r(0, 16)


@pytest.mark.parametrize("name,t", list(_layouts()), ids=[n for n, _ in _layouts()])
def test_rows_match_row_layout(fp, name, t):
    got = fp.layout_rows(t)
    lay = K.row_layout(t)
    if lay.tensor.data_ptr() != t.data_ptr() or t.ndim > 4:
        assert got is None  # the Python path copies first: the fast path declines
        return
    assert got == (lay.a, lay.b, lay.c, lay.sa, lay.sb, lay.sc, lay.col, lay.n)


def _python_linear_args(x, n, row_add):
    """What ops.linear_decode + kernels.linear_out pass, and whether they copied."""
    x2, leading = O._as_mk(x)
    m = x2.shape[0]
    copied = x2.data_ptr() != x.data_ptr() and x.numel() > 0
    srm = srn = 0
    if row_add is not None:
        expected = (n,) if leading is None else (*leading, n)
        ra = O._as_row_add(row_add, m, n, expected)
        copied = copied or ra.data_ptr() != row_add.data_ptr()
        srm = 0 if ra.shape[0] == 1 else int(ra.stride(0))
        srn = 0 if ra.shape[1] == 1 else int(ra.stride(1))
    return (m, int(x2.stride(0)), int(x2.stride(1)), srm, srn), copied


def _linear_cases():
    g = torch.Generator().manual_seed(1)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    n = 24
    xs = {
        "x1d": r(32), "x1d_strided": r(64)[::2], "x2d": r(3, 32), "x2d_t": r(32, 3).t(),
        "x2d_rows": r(6, 32)[::2], "x3d": r(2, 3, 32), "x3d_perm": r(3, 2, 32).transpose(0, 1),
    }
    for xn, x in xs.items():
        lead = tuple(x.shape[:-1])
        m = 1
        for d in lead:
            m *= d
        ras = {
            "none": None, "row_n": r(n), "row_n_strided": r(2 * n)[::2], "full": r(*lead, n),
            "m1": r(m, 1), "one_n": r(1, n), "mn_t": r(n, m).t(), "bcast3d": r(1, 1, n),
        }
        for rn, ra in ras.items():
            yield f"{xn}-{rn}", x, n, ra


@pytest.mark.parametrize("case", list(_linear_cases()), ids=[c[0] for c in _linear_cases()])
def test_linear_args_match_python_path(fp, case):
    _, x, n, ra = case
    try:
        want, copied = _python_linear_args(x, n, ra)
    except ValueError:  # row_add not broadcastable: Python raises, so the fast path must decline
        assert fp.layout_linear(x, n, ra) is None
        return
    got = fp.layout_linear(x, n, ra)
    if copied:
        assert got is None
    else:
        assert got == want
