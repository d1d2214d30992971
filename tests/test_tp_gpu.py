"""Tensor-parallel MLP kernels on the GPU.

* One GPU: every rank's shard of a layer runs through ``TPPostAttnMlp.partial``
  (the fused MLP kernels with an fp32 partial and no residual); the partials
  are summed in rank order and finished by ``residual_add_out`` -- the TP layer
  without the collective.  Compared with the oracle's partials summed the same
  way (within one bf16 rounding step: rtol 2^-7, atol 1e-3), and with the
  unsharded oracle layer within BASELINE's atol = rtol = 1e-2.
* Two or more GPUs: ranks over NCCL run chained TP layers end to end
  (``TPPostAttnMlp.__call__``, one ``all_reduce`` per layer); skipped when the
  machine has fewer than two GPUs.
"""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from oracle import fd_oracle as O

pytestmark = pytest.mark.gpu

from fused_decode_b200 import tp  # noqa: E402

TOL = {"rtol": 1e-2, "atol": 1e-2}
EPS = 1e-5


def _np(t):
    return t.detach().float().cpu().numpy()


def _layer(h, i, m, seed, dtype=torch.bfloat16, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, h, generator=g).to(dtype)
    nw = (1 + 0.1 * torch.randn(h, generator=g)).to(dtype)
    wgu = (torch.randn(2 * i, h, generator=g) * 0.02).to(dtype)
    wd = (torch.randn(h, i, generator=g) * 0.02).to(dtype)
    return [t.to(device) for t in (x, nw, wgu, wd)]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("m", [1, 4, 8])
def test_tp_shards_one_gpu(world, m):
    h, i = 1024, 2816  # i / world stays a multiple of 8 for every world here
    x, nw, wgu, wd = _layer(h, i, m, 11 + world + m)
    total = torch.zeros(m, h, device="cuda", dtype=torch.float32)
    ref_total = np.zeros((m, h), np.float32)
    for r in range(world):
        mod = tp.TPPostAttnMlp.from_full(nw, wgu, wd, r, world, EPS, kind="dot")
        part = mod.partial(x)
        assert part.dtype == torch.float32 and part.shape == (m, h)
        ref_part = O.post_attn_mlp_partial_f32(_np(x), _np(nw), _np(mod.w_gate_up), _np(mod.w_down), EPS, "bfloat16")
        torch.testing.assert_close(part.cpu(), torch.from_numpy(ref_part), rtol=1e-3, atol=1e-3)
        total += part
        ref_total += ref_part
    out = mod.finish(total, x)
    assert out.dtype == x.dtype and out.shape == x.shape and out.is_contiguous()
    full = O.post_attn_mlp(_np(x), _np(nw), _np(wgu), _np(wd), EPS, "bfloat16")
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(full), **TOL)
    # The oracle's TP emulation: the same shards' partials summed in rank order.
    # Kernel and oracle partials differ by fp32 summation order only, so the
    # two agree to one bf16 rounding step (at most 2^-7 relative; absolute near zero).
    emul = O.round_to(ref_total + _np(x), "bfloat16")
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(emul), rtol=2 ** -7, atol=1e-3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, outdir, h, i, m, layers):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        x = None
        for layer in range(layers):
            x0, nw, wgu, wd = _layer(h, i, m, 500 + layer, device=dev)
            x = x0 if x is None else x
            mod = tp.TPPostAttnMlp.from_full(nw, wgu, wd, rank, world, EPS, kind="dot")
            x = mod(x)
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"rank{rank}.npy"), _np(x))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_tp_nccl_layers():
    import torch.multiprocessing as mp

    h, i, m, layers = 1024, 2816, 4, 3
    world = min(torch.cuda.device_count(), 8)
    while (i % world or (i // world) % 8) and world > 2:  # I/world must be a multiple of 8
        world -= 1
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d, h, i, m, layers), nprocs=world, join=True,
                           start_method="spawn")
        outs = [np.load(os.path.join(d, f"rank{r}.npy")) for r in range(world)]
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])
    x = None
    for layer in range(layers):
        x0, nw, wgu, wd = [_np(t) for t in _layer(h, i, m, 500 + layer, device="cpu")]
        x = x0 if x is None else x
        x = O.post_attn_mlp(x, nw, wgu, wd, EPS, "bfloat16")
    torch.testing.assert_close(torch.from_numpy(outs[0]), torch.from_numpy(x), **TOL)
