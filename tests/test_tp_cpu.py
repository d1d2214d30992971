"""Tensor-parallel MLP host logic on CPU: sharding math and the gloo exchange.

The rank-local compute (the CUDA kernels) is replaced by the oracle here, so
these tests check what runs on the host: how ``shard_gate_up`` / ``shard_down``
cut the weights, that the per-rank fp32 partials summed by one
``all_reduce(sum)`` and added to the residual give the unsharded layer
(``post_attn_mlp_reference``, reference.py:66-79), and that a world of 2 or 4
gloo ranks agrees on the result.  Tolerance: the fp32 partials are summed in a
different order than the unsharded dot products, so the result may differ from
the unsharded oracle by one rounding step of the activation dtype; checked as
at most 1 ulp and within the parity bar atol = rtol = 1e-2.
"""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fused_decode_b200 import tp
from oracle import fd_oracle as O

H, I, M = 64, 96, 3
EPS = 1e-5


def _layer(seed, dtype=O.BF16):
    rng = np.random.default_rng(seed)

    def cast(a):
        return O.round_to(a, dtype)

    x = cast(rng.standard_normal((M, H), dtype=np.float32))
    nw = cast(1 + 0.1 * rng.standard_normal(H, dtype=np.float32))
    wgu = cast(rng.standard_normal((2 * I, H), dtype=np.float32) * np.float32(0.02))
    wd = cast(rng.standard_normal((H, I), dtype=np.float32) * np.float32(0.02))
    return x, nw, wgu, wd


def _finish(total, x, dtype):
    return O.round_to(np.asarray(total, np.float32) + x, dtype)


class OracleRank(tp.TPPostAttnMlp):
    """A TP rank whose local compute is the oracle (CPU tensors, fp32 values)."""

    dtype = O.BF16

    def partial(self, hidden2):
        p = O.post_attn_mlp_partial_f32(hidden2.numpy(), self.norm_weight.numpy(), self.w_gate_up.numpy(),
                                        self.w_down.numpy(), self.eps, self.dtype)
        return torch.from_numpy(np.ascontiguousarray(p))

    def finish(self, total, hidden2):
        return torch.from_numpy(_finish(total.numpy(), hidden2.numpy(), self.dtype))


def test_shard_bounds():
    assert tp.shard_bounds(96, 0, 2) == (0, 48)
    assert tp.shard_bounds(96, 3, 4) == (72, 96)
    with pytest.raises(ValueError):
        tp.shard_bounds(96, 2, 2)
    with pytest.raises(ValueError):
        tp.shard_bounds(100, 0, 3)


def test_shard_gate_up_restack():
    w = torch.arange(2 * I * 2, dtype=torch.float32).view(2 * I, 2)
    s = tp.shard_gate_up(w, 1, 4)
    lo, hi = I // 4, I // 2
    assert s.shape == (2 * (I // 4), 2) and s.is_contiguous()
    assert torch.equal(s[: I // 4], w[lo:hi])
    assert torch.equal(s[I // 4:], w[I + lo:I + hi])
    d = tp.shard_down(torch.arange(H * I, dtype=torch.float32).view(H, I), 2, 4)
    assert d.shape == (H, I // 4) and d.is_contiguous()
    with pytest.raises(ValueError):
        tp.shard_gate_up(w[:-1], 0, 2)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_partials_sum_to_unsharded(world):
    x, nw, wgu, wd = _layer(7)
    full = O.post_attn_mlp(x, nw, wgu, wd, EPS, O.BF16)
    total = np.zeros((M, H), np.float32)
    for r in range(world):
        g = tp.shard_gate_up(torch.from_numpy(wgu), r, world).numpy()
        d = tp.shard_down(torch.from_numpy(wd), r, world).numpy()
        total += O.post_attn_mlp_partial_f32(x, nw, g, d, EPS, O.BF16)
    got = _finish(total, x, O.BF16)
    assert np.abs(O.ulp_distance(got, full, O.BF16)).max() <= 1
    np.testing.assert_allclose(got, full, rtol=1e-2, atol=1e-2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        x = None
        for layer in range(3):  # three chained layers, every rank the same order
            x0, nw, wgu, wd = _layer(100 + layer)
            x = x0 if x is None else x
            mod = OracleRank.from_full(torch.from_numpy(nw), torch.from_numpy(wgu), torch.from_numpy(wd), rank,
                                       world, EPS)
            x = mod(torch.from_numpy(x)).numpy()
        np.save(os.path.join(outdir, f"rank{rank}.npy"), x)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_layers_gloo(world):
    """``world`` gloo ranks run three chained TP layers; every rank ends with
    the same activations, equal to the unsharded oracle chain."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d), nprocs=world, join=True,
                           start_method="spawn")
        outs = [np.load(os.path.join(d, f"rank{r}.npy")) for r in range(world)]
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])
    x = None
    for layer in range(3):
        x0, nw, wgu, wd = _layer(100 + layer)
        x = x0 if x is None else x
        x = O.post_attn_mlp(x, nw, wgu, wd, EPS, O.BF16)
    assert np.abs(O.ulp_distance(outs[0], x, O.BF16)).max() <= 2
    np.testing.assert_allclose(outs[0], x, rtol=1e-2, atol=1e-2)
