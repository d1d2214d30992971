"""Tensor-parallel MLP kernels on the GPU.

* One GPU: every rank's shard of a layer runs through ``TPPostAttnMlp.partial``
  (the fused MLP kernels with an fp32 partial and no residual); the partials
  are summed in rank order and finished by ``residual_add_out`` -- the TP layer
  without the collective.  Compared with the oracle's partials summed the same
  way (within one bf16 rounding step: rtol 2^-7, atol 1e-3), and with the
  unsharded oracle layer within the parity bar atol = rtol = 1e-2.
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


def _rope_tables(positions, dim, theta=500000.0):
    inv = theta ** (-torch.arange(0, dim, 2, dtype=torch.float32) / dim)
    f = torch.outer(torch.arange(positions, dtype=torch.float32), inv)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


@pytest.mark.parametrize("m", [1, 4, 8])
def test_tp_decode_block_llama70b(m):
    """The tensor-parallel decode block at full Llama-3-70B widths (hidden 8192, intermediate
    28672, 64 query / 8 KV heads of 128): add_rms_norm, RoPE on q and k, then
    the MLP with gate/up column-sharded and down row-sharded over 8 emulated
    ranks on one GPU (the allreduce is the fp32 sum of the rank partials), then
    the residual add.  Every stage against the oracle at atol = rtol = 1e-2."""
    from fused_decode_b200 import add_rms_norm, rope

    h, i, world, eps = 8192, 28672, 8, 1e-5
    g = torch.Generator(device="cpu").manual_seed(70 + m)
    bf = torch.bfloat16
    x = torch.randn(m, h, generator=g).to(bf).cuda()
    res = torch.randn(m, h, generator=g).to(bf).cuda()
    attn_w = (1 + 0.1 * torch.randn(h, generator=g)).to(bf).cuda()
    q = torch.randn(m, 1, 64, 128, generator=g).to(bf).cuda()
    k = torch.randn(m, 1, 8, 128, generator=g).to(bf).cuda()
    cos, sin = _rope_tables(1024, 128)
    pos = torch.randint(0, 1024, (m,), generator=g)
    cos_b = cos[pos].view(m, 1, 1, 128).cuda()
    sin_b = sin[pos].view(m, 1, 1, 128).cuda()
    # random-init layer weights, N(0, 0.02)
    mlp_w = (1 + 0.1 * torch.randn(h, generator=g)).to(bf).cuda()
    wgu = torch.empty(2 * i, h, dtype=bf, device="cuda")
    wd = torch.empty(h, i, dtype=bf, device="cuda")
    gd = torch.Generator(device="cuda").manual_seed(700 + m)
    for r0 in range(0, 2 * i, 8192):  # chunked to bound the fp32 temporary
        wgu[r0:r0 + 8192] = (torch.randn(min(8192, 2 * i - r0), h, device="cuda", generator=gd) * 0.02).to(bf)
    for r0 in range(0, h, 2048):
        wd[r0:r0 + 2048] = (torch.randn(2048, i, device="cuda", generator=gd) * 0.02).to(bf)

    # stage 1: add_rms_norm (attention-out residual) and RoPE on q/k
    normed, hidden = add_rms_norm(x, res, attn_w, eps)
    ref_normed, ref_hidden = O.add_rms_norm(_np(x), _np(res), _np(attn_w), eps, "bfloat16")
    torch.testing.assert_close(normed.float().cpu(), torch.from_numpy(ref_normed), **TOL)
    torch.testing.assert_close(hidden.float().cpu(), torch.from_numpy(ref_hidden), **TOL)
    for t in (q, k):
        out = rope(t, cos_b, sin_b)
        ref = O.rope(_np(t), _np(cos_b), _np(sin_b), "bfloat16")
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(ref), **TOL)

    # stage 2: tensor-parallel MLP, ranks emulated in order on one GPU
    total = torch.zeros(m, h, device="cuda", dtype=torch.float32)
    for r in range(world):
        mod = tp.TPPostAttnMlp.from_full(mlp_w, wgu, wd, r, world, eps, kind="dot")
        total += mod.partial(hidden)
    out = mod.finish(total, hidden)
    ref = O.post_attn_mlp(_np(hidden), _np(mlp_w), _np(wgu), _np(wd), eps, "bfloat16")
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(ref), **TOL)


@pytest.mark.parametrize("fold", ["1", "0"])
@pytest.mark.parametrize("h", [1024, 4096])
@pytest.mark.parametrize("m", [1, 5, 16])
def test_tp_exchange_single_rank(m, h, fold, monkeypatch):
    """The NVLink-exchange layer (down-projection partials published into the
    exchange buffer; the rank sum in a separate kernel, or with FD_TP_FOLD=1
    in the down projection's epilogue) with a group of one: equal bit for bit
    to post_attn_mlp, round after round (the buffer's two parities
    alternate), inside a CUDA graph too, and the status word stays clear.
    h = 1024 splits the down projection stream-K, h = 4096 by clusters."""
    from fused_decode_b200 import kernels as K
    from fused_decode_b200 import post_attn_mlp
    from fused_decode_b200.stack import MlpStack

    monkeypatch.setenv("FD_TP_FOLD", fold)
    i = 2816
    ex = tp.TPExchange(h, m_max=16)
    try:
        layers = [_layer(h, i, m, 900 + l)[1:] for l in range(3)]
        x0 = _layer(h, i, m, 950)[0]
        x = x0
        for rnd in range(5):  # several rounds on the same buffer
            nw, wgu, wd = layers[rnd % 3]
            mod = tp.TPPostAttnMlp(nw, wgu, wd, EPS, kind="dot", exchange=ex)
            got = mod(x)
            want = post_attn_mlp(x, nw, wgu, wd, EPS, kind="dot")
            assert torch.equal(got, want), rnd
            # each round within the parity bar of the oracle on its own input
            ref = O.post_attn_mlp(_np(x), _np(nw), _np(wgu), _np(wd), EPS, "bfloat16")
            torch.testing.assert_close(got.float().cpu(), torch.from_numpy(ref), **TOL)
            x = got

        def fn(t, nw, wgu, wd):
            return tp.TPPostAttnMlp(nw, wgu, wd, EPS, kind="dot", exchange=ex)(t)

        stack = MlpStack(layers, m, EPS, kind="dot", layer_fn=fn)
        a = stack(x0).clone()
        b = stack(x0).clone()
        assert torch.equal(a, b)
        y = x0
        for nw, wgu, wd in layers:
            y = post_attn_mlp(y, nw, wgu, wd, EPS, kind="dot")
        assert torch.equal(a, y)
        torch.cuda.synchronize()
        assert all(v == 0 for v in K.WORKSPACES.status().values()), K.WORKSPACES.status()
    finally:
        ex.close()


@pytest.mark.parametrize("fold", ["0", "1"])
def test_tp_exchange_single_rank_streamed(fold, monkeypatch):
    """A tensor-parallel layer (group of one) whose gate/up stage streams the
    normalised rows (8 rows at 70B hidden width take that mode by default):
    the same bits as post_attn_mlp, round after round, within the parity bar
    of the oracle, four launches a layer with the reduce kernel."""
    from fused_decode_b200 import kernels as K
    from fused_decode_b200 import post_attn_mlp
    from fused_decode_b200.stack import MlpStack

    monkeypatch.setenv("FD_TP_FOLD", fold)
    h, i, m = 8192, 2816, 8
    ex = tp.TPExchange(h, m_max=16)
    try:
        layers = [_layer(h, i, m, 1500 + l)[1:] for l in range(2)]
        x = _layer(h, i, m, 1550)[0]
        for rnd in range(4):
            nw, wgu, wd = layers[rnd % 2]
            got = tp.TPPostAttnMlp(nw, wgu, wd, EPS, kind="dot", exchange=ex)(x)
            assert torch.equal(got, post_attn_mlp(x, nw, wgu, wd, EPS, kind="dot")), rnd
            ref = O.post_attn_mlp(_np(x), _np(nw), _np(wgu), _np(wd), EPS, "bfloat16")
            torch.testing.assert_close(got.float().cpu(), torch.from_numpy(ref), **TOL)
            x = got
        per_layer = 3 if fold == "1" else 4
        assert MlpStack(layers, m, EPS, kind="dot", exchange=ex).launches_per_replay == per_layer * len(layers)
        torch.cuda.synchronize()
        assert all(v == 0 for v in K.WORKSPACES.status().values()), K.WORKSPACES.status()
    finally:
        ex.close()


@pytest.mark.parametrize("m", [1, 8])
def test_tp_exchange_modes_interleaved(m, monkeypatch):
    """Layers alternating between the folded rank sum and the separate reduce
    kernel on one exchange buffer (group of one): both advance the same round
    number, so every layer matches post_attn_mlp bit for bit, and the stack
    entry point enqueues two launches per layer folded, three otherwise."""
    from fused_decode_b200 import kernels as K
    from fused_decode_b200 import post_attn_mlp
    from fused_decode_b200.stack import MlpStack

    h, i = 4096, 2816
    ex = tp.TPExchange(h, m_max=16)
    try:
        layers = [_layer(h, i, m, 1200 + l)[1:] for l in range(2)]
        x = _layer(h, i, m, 1250)[0]
        for rnd in range(6):
            monkeypatch.setenv("FD_TP_FOLD", "01"[rnd % 2])
            nw, wgu, wd = layers[rnd % 2]
            got = tp.TPPostAttnMlp(nw, wgu, wd, EPS, kind="dot", exchange=ex)(x)
            assert torch.equal(got, post_attn_mlp(x, nw, wgu, wd, EPS, kind="dot")), rnd
            x = got
        for fold, per_layer in (("1", 2), ("0", 3)):
            monkeypatch.setenv("FD_TP_FOLD", fold)
            assert MlpStack(layers, m, EPS, kind="dot", exchange=ex).launches_per_replay == per_layer * len(layers)
        torch.cuda.synchronize()
        assert all(v == 0 for v in K.WORKSPACES.status().values()), K.WORKSPACES.status()
    finally:
        ex.close()


def _rank_main_nvlink(rank, world, port, outdir, h, i, m, layers):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        dev = torch.device("cuda", rank)
        ex = tp.TPExchange(h, m_max=16)
        res = []
        # rank sum in the down epilogue, then as its own kernel; then with the
        # gate/up stage streaming the normalised rows
        for fold, stream in (("1", "0"), ("0", "0"), ("0", "1")):
            os.environ["FD_TP_FOLD"] = fold
            os.environ["FD_GATEUP_STREAM"] = stream
            x, outs = None, []
            for layer in range(layers):
                x0, nw, wgu, wd = _layer(h, i, m, 500 + layer, device=dev)
                x = x0 if x is None else x
                x = tp.TPPostAttnMlp.from_full(nw, wgu, wd, rank, world, EPS, kind="dot", exchange=ex)(x)
                outs.append(_np(x))
            res.append(np.stack(outs))
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"rank{rank}.npy"), np.stack(res))  # [mode, layer, m, h]
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_tp_nvlink_layers():
    """Chained tensor-parallel layers with the NVLink exchange on 2..8 GPUs,
    the rank sum folded into the down projection and as its own kernel, and
    the gate/up stage streaming the normalised rows: every rank ends with the
    same bits in every mode, each layer within the parity bar of the
    unsharded oracle on its own input.  h = 1024 splits the down projection stream-K, h = 4096 by
    clusters."""
    import torch.multiprocessing as mp

    for h in (1024, 4096):
        _nvlink_layers(h)


def _nvlink_layers(h):
    import torch.multiprocessing as mp

    i, m, layers = 2816, 4, 3
    world = min(torch.cuda.device_count(), 8)
    while (i % world or (i // world) % 8) and world > 2:
        world -= 1
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main_nvlink, args=(world, _free_port(), d, h, i, m, layers), nprocs=world,
                           join=True, start_method="spawn")
        outs = [np.load(os.path.join(d, f"rank{r}.npy")) for r in range(world)]
    for o in outs:
        for mode in range(o.shape[0]):
            assert np.array_equal(o[mode], outs[0][0]), mode
    # every layer within the parity bar of the unsharded oracle on its own input
    x = None
    for layer in range(layers):
        x0, nw, wgu, wd = [_np(t) for t in _layer(h, i, m, 500 + layer, device="cpu")]
        x = x0 if x is None else outs[0][0][layer - 1]
        ref = O.post_attn_mlp(x, nw, wgu, wd, EPS, "bfloat16")
        torch.testing.assert_close(torch.from_numpy(outs[0][0][layer]), torch.from_numpy(ref), **TOL)


@pytest.mark.parametrize("m", [1, 8])
def test_tp_stack_single_rank(m, monkeypatch):
    """The tensor-parallel stack entry point (one persistent kernel: gate/up,
    down with the partials published into the exchange buffer, reduce) with a
    group of one: the same bits as per-layer calls, replay after replay in a
    CUDA graph (the exchange rounds advance), each layer within the parity bar
    of the oracle on its own input, and the per-layer exchange path still in
    step with the round number afterwards."""
    from fused_decode_b200 import kernels as K
    from fused_decode_b200 import post_attn_mlp
    from fused_decode_b200.stack import MlpStack

    h, i, layers = 1024, 2816, 4
    monkeypatch.setenv("FD_STACK_PERSISTENT", "1")
    monkeypatch.setenv("FD_GEMV_CLUSTER", "0")
    ex = tp.TPExchange(h, m_max=16)
    try:
        ws = [_layer(h, i, m, 960 + l)[1:] for l in range(layers)]
        x0 = _layer(h, i, m, 990)[0]
        out = torch.empty_like(x0)
        K.post_attn_mlp_tp_stack_out(x0, ws, out, EPS, "dot", ex)
        x = x0
        for nw, wgu, wd in ws:
            y = post_attn_mlp(x, nw, wgu, wd, EPS, kind="dot")
            torch.testing.assert_close(y.float().cpu(), torch.from_numpy(
                O.post_attn_mlp(_np(x), _np(nw), _np(wgu), _np(wd), EPS, "bfloat16")), **TOL)
            x = y
        assert torch.equal(out, x)
        stack = MlpStack(ws, m, EPS, kind="dot", exchange=ex)
        assert stack.launches_per_replay == 1
        for _ in range(3):
            assert torch.equal(stack(x0), x)
        assert torch.equal(tp.TPPostAttnMlp(*ws[0], EPS, kind="dot", exchange=ex)(x0),
                           post_attn_mlp(x0, *ws[0], EPS, kind="dot"))
        torch.cuda.synchronize()
        assert all(v == 0 for v in K.WORKSPACES.status().values()), K.WORKSPACES.status()
    finally:
        ex.close()


def _rank_main_tp_stack(rank, world, port, outdir, h, i, m, layers):
    import torch.distributed as dist

    from fused_decode_b200 import kernels as K
    from fused_decode_b200.stack import MlpStack

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["FD_STACK_PERSISTENT"] = "1"  # the persistent kernel, in this rank process only
    os.environ["FD_GEMV_CLUSTER"] = "0"  # and the per-layer path split stream-K as the kernel splits it
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        dev = torch.device("cuda", rank)
        ex = tp.TPExchange(h, m_max=16)
        shards, x0 = [], None
        for layer in range(layers):
            xl, nw, wgu, wd = _layer(h, i, m, 500 + layer, device=dev)
            x0 = xl if x0 is None else x0
            shards.append((nw, tp.shard_gate_up(wgu, rank, world), tp.shard_down(wd, rank, world)))
        out = torch.empty_like(x0)
        K.post_attn_mlp_tp_stack_out(x0, shards, out, EPS, "dot", ex)  # one persistent kernel
        x = x0
        for nw, wgu, wd in shards:  # two launches per layer
            x = tp.TPPostAttnMlp(nw, wgu, wd, EPS, kind="dot", exchange=ex)(x)
        stack = MlpStack(shards, m, EPS, kind="dot", exchange=ex)
        g = [stack(x0).clone() for _ in range(2)]
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"rank{rank}.npy"),
                np.stack([_np(out), _np(x), _np(g[0]), _np(g[1])]))
        dist.barrier()
        del stack
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_tp_stack_nvlink():
    """The persistent tensor-parallel stack on 2..8 GPUs: on every rank the
    same bits as the per-layer NVLink path and as its own graph replays, and
    equal across ranks; the chain matches the unsharded oracle chain."""
    import torch.multiprocessing as mp

    h, i, m, layers = 1024, 2816, 4, 3
    world = min(torch.cuda.device_count(), 8)
    while (i % world or (i // world) % 8) and world > 2:
        world -= 1
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main_tp_stack, args=(world, _free_port(), d, h, i, m, layers), nprocs=world,
                           join=True, start_method="spawn")
        outs = [np.load(os.path.join(d, f"rank{r}.npy")) for r in range(world)]
    for o in outs:
        assert np.array_equal(o[0], o[1]) and np.array_equal(o[0], o[2]) and np.array_equal(o[0], o[3])
        assert np.array_equal(o[0], outs[0][0])
    x = None
    for layer in range(layers):
        x0, nw, wgu, wd = [_np(t) for t in _layer(h, i, m, 500 + layer, device="cpu")]
        x = x0 if x is None else x
        x = O.post_attn_mlp(x, nw, wgu, wd, EPS, "bfloat16")
    torch.testing.assert_close(torch.from_numpy(outs[0][0]), torch.from_numpy(x), rtol=2e-2, atol=2e-2)
