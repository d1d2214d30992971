"""The strided-row contract on CPU: kernels.row_layout describes a tensor the
way the reference's row_layout does (kernels.py:26-88): up to three leading
dims right-aligned into (a, b, c) with their strides, the last-dim stride and
the row length; more than four dims or a negative stride go through a
contiguous copy first."""

import pytest
import torch

from fused_decode_b200 import kernels as K


def _fields(l):
    return (l.a, l.b, l.c, l.sa, l.sb, l.sc, l.col, l.n)


def test_one_to_four_dims():
    assert _fields(K.row_layout(torch.empty(7))) == (1, 1, 1, 0, 0, 0, 1, 7)
    assert _fields(K.row_layout(torch.empty(3, 5))) == (1, 1, 3, 0, 0, 5, 1, 5)
    assert _fields(K.row_layout(torch.empty(2, 3, 5))) == (1, 2, 3, 0, 15, 5, 1, 5)
    assert _fields(K.row_layout(torch.empty(4, 2, 3, 5))) == (4, 2, 3, 30, 15, 5, 1, 5)


def test_strided_views_keep_their_strides():
    x = torch.empty(6, 10)
    left = x[:, :4]  # row stride 10, unit column stride
    assert _fields(K.row_layout(left)) == (1, 1, 6, 0, 0, 10, 1, 4)
    t = torch.empty(5, 3).t()  # shape (3, 5), strides (1, 3)
    assert _fields(K.row_layout(t)) == (1, 1, 3, 0, 0, 1, 3, 5)
    q = torch.empty(1, 2048, 32, 128).transpose(1, 2)  # (1, 32, 2048, 128)
    lay = K.row_layout(q)
    assert (lay.a, lay.b, lay.c, lay.n) == (1, 32, 2048, 128)
    assert (lay.sb, lay.sc, lay.col) == (128, 32 * 128, 1)


def test_broadcast_stride_zero():
    cos = torch.empty(2048, 1, 128).expand(2048, 32, 128)
    assert _fields(K.row_layout(cos)) == (1, 2048, 32, 0, 128, 0, 1, 128)


def test_five_dims_and_negative_strides_copy():
    x5 = torch.arange(2 * 3 * 4 * 5 * 6, dtype=torch.float32).view(2, 3, 4, 5, 6)
    lay = K.row_layout(x5)
    assert _fields(lay) == (1, 1, 120, 0, 0, 6, 1, 6)
    assert torch.equal(lay.tensor.view(x5.shape), x5)
    flipped = torch.arange(12, dtype=torch.float32).view(3, 4).flip(0)
    lay = K.row_layout(flipped)
    assert lay.tensor.is_contiguous() and torch.equal(lay.tensor, flipped)


def test_zero_dim_rejected_and_grid_checks():
    with pytest.raises(ValueError):
        K.row_layout(torch.tensor(1.0))
    a = K.row_layout(torch.empty(3, 5))
    b = K.row_layout(torch.empty(3, 6))
    with pytest.raises(ValueError):
        K._same_grid(a, b, "out")
    assert not K._runnable(K.row_layout(torch.empty(0, 5)))
    assert K._runnable(a)
