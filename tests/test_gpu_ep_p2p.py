"""Device-initiated expert-parallel exchange (include/nvfp4_ep.h): dispatch
and combine kernels that store and load rows in the ranks' windows, ordered
by flags with bounded waits.

On one GPU the ranks are emulated in one process: each rank has its own
window on the device, and the ranks' steps run one after another in one
stream (every rank's dispatch, then every rank's wait, experts, done signal
and combine), so every wait finds its flags already raised.  Each rank's
output must equal the single-GPU layer's on the same tokens bit for bit
(the expert rows are the same arithmetic, the combine sums the same rows in
the same slot order).  The timeout tests leave one flag unraised and check
that the wait gives up, records the missing rank and leaves the context
usable.  The 2-process test runs the real exchange over NVLink when the host
has 2 or 4 GPUs (one process per GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

E, H, I, K, T = 16, 256, 256, 4, 8  # the grouped-GEMV expert path on every rank count


def moe_dict(seed=11):
    from nvfp4 import synthetic

    return synthetic.moe_weights(E, H, I, seed=seed)


def local_weights(wd, rank, world):
    from nvfp4.moe import MoEWeights

    epr = E // world
    sl = slice(rank * epr, (rank + 1) * epr)
    return MoEWeights.from_dict({k: (v[sl] if k != "router" else v) for k, v in wd.items()})


def tokens(seed, n=T):
    from nvfp4 import synthetic

    x = synthetic.bf16_round(synthetic.activations(n, H, seed=seed))
    return torch.from_numpy(x).cuda().to(torch.bfloat16)


def emulated_step(pws, full, locs, xs, res):
    """One step of every rank, the ranks' launches interleaved phase by phase."""
    from nvfp4 import ep
    from nvfp4.moe import moe_route

    world = len(pws)
    epr = E // world
    routes = [moe_route(full, x, top_k=K)[:2] for x in xs]
    for r in range(world):
        ep.p2p_dispatch(pws[r], routes[r][0], xs[r], epr)
    for r in range(world):
        ep.p2p_wait_dispatch(pws[r])
    for r in range(world):
        ep.p2p_experts(pws[r], locs[r], xs[r].shape[0], K)
    for r in range(world):
        ep.p2p_signal_done(pws[r])
    return [ep.p2p_combine(pws[r], routes[r][0], routes[r][1], epr, residual=res[r])
            for r in range(world)]


@pytest.mark.parametrize("world", [1, 2, 4])
def test_emulated_ranks_equal_single_gpu(cuda, world):
    from nvfp4.ep import PeerWindows
    from nvfp4.moe import MoELayer, MoEWeights

    wd = moe_dict()
    full = MoEWeights.from_dict(wd)
    layer = MoELayer(full, top_k=K)
    locs = [local_weights(wd, r, world) for r in range(world)]
    pws = PeerWindows.emulated(world, T * K, H)
    try:
        for step in range(3):  # the step counters advance; windows are reused
            n = T if step < 2 else T // 2  # a smaller step inside the same windows
            xs = [tokens(100 * step + r, n) for r in range(world)]
            res = [tokens(1000 + 100 * step + r, n) for r in range(world)]
            ys = emulated_step(pws, full, locs, xs, res)
            for r in range(world):
                ref = layer(xs[r], residual=res[r])
                assert torch.equal(ys[r].view(torch.int16), ref.view(torch.int16)), (step, r)
        torch.cuda.synchronize()
        assert all(pw.error() == 0 for pw in pws)
    finally:
        pws[0].close()


def test_single_rank_layer_forward(cuda):
    """EPMoELayer(exchange="p2p") with one rank (no process group): the
    whole step in one call, fp32 and bf16 outputs, against the single-GPU
    layer."""
    from nvfp4.ep import EPMoELayer
    from nvfp4.moe import MoELayer, MoEWeights

    wd = moe_dict()
    full = MoEWeights.from_dict(wd)
    ep_layer = EPMoELayer(full, full.router, top_k=K, num_experts=E, exchange="p2p",
                          max_tokens=T)
    try:
        for step in range(2):
            x, res = tokens(7 + step), tokens(70 + step)
            ref = MoELayer(full, top_k=K)(x, residual=res)
            got = ep_layer(x, residual=res)
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
            ref32 = MoELayer(full, top_k=K)(x, out=torch.empty((T, H), device="cuda"))
            got32 = ep_layer.forward_p2p(x, out=torch.empty((T, H), device="cuda"))
            assert torch.equal(got32, ref32)
        assert ep_layer.windows.error() == 0
        with pytest.raises(ValueError):
            ep_layer(tokens(1, T + 1))
    finally:
        ep_layer.close()


def test_layers_share_windows(cuda):
    """Two layers of a stack on one set of windows (the step counter runs on
    across layers): equal to the two single-GPU layers applied in turn."""
    from nvfp4.ep import EPMoELayer, PeerWindows
    from nvfp4.moe import MoELayer, MoEWeights

    ws = [MoEWeights.from_dict(moe_dict(seed)) for seed in (11, 12)]
    pw = PeerWindows.rendezvous(T * K, H)
    layers = [EPMoELayer(w, w.router, top_k=K, num_experts=E, exchange="p2p", max_tokens=T,
                         windows=pw) for w in ws]
    try:
        with pytest.raises(ValueError):
            EPMoELayer(ws[0], ws[0].router, top_k=K, num_experts=E, exchange="p2p",
                       max_tokens=2 * T, windows=pw)
        for step in range(2):
            h = tokens(50 + step)
            ref = h
            for lyr, w in zip(layers, ws):
                h = lyr(h, residual=h)
                ref = MoELayer(w, top_k=K)(ref, residual=ref)
                assert torch.equal(h.view(torch.int16), ref.view(torch.int16)), step
        assert pw.error() == 0
    finally:
        for lyr in layers:
            lyr.close()  # shared windows stay open
        pw.close()


def test_dispatch_wait_times_out(cuda):
    """Rank 1 never dispatches: rank 0's wait gives up after its bound,
    records rank 1 as missing, and the context stays usable."""
    from nvfp4 import _lib, ep
    from nvfp4.moe import MoEWeights, moe_route

    wd = moe_dict()
    full = MoEWeights.from_dict(wd)
    pws = ep.PeerWindows.emulated(2, T * K, H, timeout_ms=20)
    try:
        x = tokens(3)
        ids, _, _ = moe_route(full, x, top_k=K)
        ep.p2p_dispatch(pws[0], ids, x, E // 2)
        ep.p2p_wait_dispatch(pws[0])
        torch.cuda.synchronize()
        err = pws[0].error()
        assert err == _lib.EP_ERR_DISPATCH_TIMEOUT | (1 << (8 + 1))
        assert pws[0].error() == 0  # cleared by the first read
        assert torch.cuda.is_available() and float(torch.ones(4, device="cuda").sum()) == 4.0
    finally:
        pws[0].close()


def test_ranks_with_different_token_counts_are_reported(cuda):
    """The window layout puts source rank r's slots at r*T*k, so every rank
    must step with the same T.  Rank 1 dispatches half as many tokens as rank
    0 (every row still inside the windows): each rank's wait records the
    other as a shape mismatch."""
    from nvfp4 import _lib, ep
    from nvfp4.moe import MoEWeights, moe_route

    full = MoEWeights.from_dict(moe_dict())
    pws = ep.PeerWindows.emulated(2, T * K, H)
    try:
        xs = [tokens(21), tokens(22, T // 2)]
        for r in range(2):
            ids, _, _ = moe_route(full, xs[r], top_k=K)
            ep.p2p_dispatch(pws[r], ids, xs[r], E // 2)
        for r in range(2):
            ep.p2p_wait_dispatch(pws[r])
        torch.cuda.synchronize()
        assert pws[0].error() == _lib.EP_ERR_SHAPE | (1 << (8 + 1))
        assert pws[1].error() == _lib.EP_ERR_SHAPE | (1 << (8 + 0))
    finally:
        pws[0].close()


def test_combine_wait_times_out(cuda):
    """Rank 1 dispatches but never signals its experts done: rank 0's
    combine gives up, records rank 1, and leaves its output untouched."""
    from nvfp4 import _lib, ep
    from nvfp4.moe import MoEWeights, moe_route

    wd = moe_dict()
    full = MoEWeights.from_dict(wd)
    locs = [local_weights(wd, r, 2) for r in range(2)]
    pws = ep.PeerWindows.emulated(2, T * K, H, timeout_ms=20)
    try:
        xs = [tokens(5), tokens(6)]
        routes = [moe_route(full, x, top_k=K)[:2] for x in xs]
        for r in range(2):
            ep.p2p_dispatch(pws[r], routes[r][0], xs[r], E // 2)
        for r in range(2):
            ep.p2p_wait_dispatch(pws[r])
        ep.p2p_experts(pws[0], locs[0], T, K)
        ep.p2p_signal_done(pws[0])
        sentinel = torch.full((T, H), 7.0, dtype=torch.bfloat16, device="cuda")
        y = ep.p2p_combine(pws[0], routes[0][0], routes[0][1], E // 2, out=sentinel.clone())
        torch.cuda.synchronize()
        assert pws[0].error() == _lib.EP_ERR_DONE_TIMEOUT | (1 << (8 + 1))
        assert pws[1].error() == 0
        assert torch.equal(y, sentinel)
    finally:
        pws[0].close()


def _worker(rank, world, port, ret):
    import datetime
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nvfp4-mojo_b200"))
    sys.path.insert(0, str(root))
    import torch.distributed as dist
    from nvfp4.ep import EPMoELayer

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    layer = None
    try:
        wd = moe_dict()
        local = local_weights(wd, rank, world)
        layer = EPMoELayer(local, local.router, top_k=K, num_experts=E, exchange="p2p",
                           max_tokens=T, timeout_ms=5000)
        outs = []
        for step in range(3):
            x, res = tokens(100 * step + rank), tokens(1000 + 100 * step + rank)
            outs.append(layer(x, residual=res).view(torch.int16).cpu().numpy().tolist())
        ret[rank] = outs
        # The step replayed from a CUDA graph (no host work between launches).
        x, res = tokens(rank), tokens(1000 + rank)
        y_eager = layer(x, residual=res)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            yg = layer(x, residual=res)
        dist.barrier()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        ret[f"graph{rank}"] = bool(torch.equal(yg, y_eager))
        ret[f"err{rank}"] = layer.windows.error()
        del g
        dist.barrier()
    finally:
        if layer is not None:
            torch.cuda.synchronize()
            dist.barrier()  # no peer still reads this rank's window
            layer.close()
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4])
def test_p2p_multi_gpu_equals_single_gpu(cuda, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from nvfp4.moe import MoELayer, MoEWeights

    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), ret), nprocs=world, join=True)
    layer = MoELayer(MoEWeights.from_dict(moe_dict()), top_k=K)
    for r in range(world):
        assert ret[f"graph{r}"] and ret[f"err{r}"] == 0
        for step in range(3):
            x, res = tokens(100 * step + r), tokens(1000 + 100 * step + r)
            ref = layer(x, residual=res).view(torch.int16).cpu().numpy()
            assert np.array_equal(np.array(ret[r][step], np.int16), ref), (r, step)
