"""Expert-parallel MoE exchange logic on CPU ranks (torch.distributed gloo,
world size 2): the EPMoELayer host algorithm (route -> dispatch plan ->
count / row / expert-id all-to-all -> local experts -> reverse all-to-all ->
combine in slot order), in both exchange modes (variable counts, and fixed
capacity with padded rows), with a CPU backend whose arithmetic is the
oracle's.  The result must equal the single-process oracle MoE on the same
tokens."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

E, H, I, K_TOP = 8, 128, 128, 2


class CpuBackend:
    """Oracle arithmetic for the per-rank steps (test infrastructure)."""

    def __init__(self, wd, rank, world):
        from oracle import oracle as O

        self.O = O
        self.wd = wd
        self.epr = E // world
        self.lo = rank * self.epr

    def route(self, x):
        xs = x.float().numpy()
        _, ids, tw = self.O.moe(xs, self.wd, top_k=K_TOP)  # oracle routing (+ outputs unused)
        return torch.from_numpy(ids), torch.from_numpy(tw)

    def plan(self, ids, epr, world):
        flat = ids.reshape(-1).numpy()
        dst = flat // epr
        order = np.argsort(dst, kind="stable")
        counts = np.bincount(dst, minlength=world).astype(np.int32)
        slot_pos = np.empty_like(order)
        slot_pos[order] = np.arange(len(order))
        return (torch.from_numpy(counts), torch.from_numpy((order // K_TOP).astype(np.int32)),
                torch.from_numpy((flat[order] % epr).astype(np.int32)),
                torch.from_numpy(slot_pos.astype(np.int32)))

    def gather(self, x, idx):
        return x[idx.long()]

    def pad(self, x, counts, send_token, send_expert, slot_pos, cap, world):
        """Numpy restatement of nvfp4_ep_dispatch_padded."""
        c = counts.numpy()
        off = np.concatenate([[0], np.cumsum(c)[:-1]])
        rows = torch.zeros((world * cap, x.shape[1]), dtype=x.dtype)
        rows_e = torch.full((world * cap,), -1, dtype=torch.int32)
        for r in range(world):
            for p in range(min(int(c[r]), cap)):
                i = off[r] + p
                rows[r * cap + p] = x[int(send_token[i])]
                rows_e[r * cap + p] = send_expert[i]
        sp = slot_pos.numpy()
        slot_pad = np.full(sp.shape, -1, np.int32)
        for s_, i in enumerate(sp):
            if i >= 0:
                r = int(np.searchsorted(np.cumsum(c), i, side="right"))
                slot_pad[s_] = r * cap + (i - off[r])
        return rows, rows_e, torch.from_numpy(slot_pad)

    def experts(self, rows, local_ids):
        O, wd = self.O, self.wd
        out = np.zeros((rows.shape[0], H), np.float32)
        xs = rows.float().numpy()
        for r, le in enumerate(local_ids.numpy()):
            if le < 0:
                continue  # padding row
            e = self.lo + int(le)
            h = O.matvec(wd["gu_w"][e], wd["gu_sf"][e], xs[r], ws2_rows=wd["gu_ws2"][e])
            a = np.array([O.silu(float(v)) for v in h[:I]], np.float32) * h[I:]
            out[r] = O.matvec(wd["dn_w"][e], wd["dn_sf"][e], a, ws2_rows=wd["dn_ws2"][e])
        return torch.from_numpy(out)

    def combine(self, y_send, tw, slot_pos, residual):
        T = tw.shape[0]
        y = np.zeros((T, H), np.float32)
        ys, w, sp = y_send.numpy(), tw.numpy(), slot_pos.numpy()
        for t in range(T):
            for j in range(K_TOP):
                y[t] += w[t, j] * ys[sp[t * K_TOP + j]]
        return torch.from_numpy(y)


def _worker(rank, world, port, static, ret):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nvfp4-mojo_b200"))
    sys.path.insert(0, str(root))
    import torch.distributed as dist
    from nvfp4 import synthetic
    from nvfp4.ep import EPMoELayer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wd = synthetic.moe_weights(E, H, I, seed=5)
        x_all = synthetic.bf16_round(synthetic.activations(6 * world, H, seed=6))
        x = torch.from_numpy(x_all[6 * rank:6 * (rank + 1)])
        layer = EPMoELayer(None, torch.from_numpy(wd["router"]), top_k=K_TOP, num_experts=E,
                           backend=CpuBackend(wd, rank, world), static=static)
        assert layer.uses_static(x.shape[0]) == static
        y = layer(x).numpy()
        ret[rank] = y.tolist()
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("static", [False, True])
def test_ep_exchange_matches_single_process_oracle(O, static):
    from nvfp4 import synthetic

    world = 2
    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), static, ret), nprocs=world, join=True)
    wd = synthetic.moe_weights(E, H, I, seed=5)
    x_all = synthetic.bf16_round(synthetic.activations(6 * world, H, seed=6))
    ref, _, _ = O.moe(x_all, wd, top_k=K_TOP)
    got = np.concatenate([np.array(ret[r], np.float32) for r in range(world)])
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def _handles_worker(rank, world, port, ret):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nvfp4-mojo_b200"))
    import torch.distributed as dist
    from nvfp4.ep import exchange_handles

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes((rank * 37 + i) % 256 for i in range(64))
        ret[rank] = [list(h) for h in exchange_handles(mine)]
    finally:
        dist.destroy_process_group()


def test_peer_window_handle_exchange():
    """exchange_handles: every rank gets every rank's 64-byte IPC handle, in
    rank order (gloo ranks stand in for the GPUs' processes)."""
    world = 3
    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    mp.spawn(_handles_worker, args=(world, _port(), ret), nprocs=world, join=True)
    want = [[(p * 37 + i) % 256 for i in range(64)] for p in range(world)]
    for r in range(world):
        assert ret[r] == want


def peer_step_model(O, wd, xs, world, k):
    """The peer-exchange step (include/nvfp4_ep.h) with numpy arrays for the
    windows: each rank's dispatch stores row x[t] and the local expert id at
    row rank*T*k + s of the owner's window (id -1 in the others), each owner
    runs its experts on its world*T*k rows, each rank combines its slots from
    the owners' output rows in j order."""
    T = xs[0].shape[0]
    R, epr = T * k, E // world
    recv_x = [np.zeros((world * R, H), np.float32) for _ in range(world)]
    recv_e = [np.full(world * R, -1, np.int64) for _ in range(world)]
    routes = []
    for r in range(world):
        _, ids, tw = O.moe(xs[r], wd, top_k=k)
        routes.append((ids, tw))
        for s, e in enumerate(ids.reshape(-1)):
            d = int(e) // epr
            recv_x[d][r * R + s] = xs[r][s // k]
            recv_e[d][r * R + s] = int(e) % epr
    out = [np.zeros((world * R, H), np.float32) for _ in range(world)]
    for d in range(world):
        for row in range(world * R):
            le = recv_e[d][row]
            if le < 0:
                continue
            e = d * epr + le
            h = O.matvec(wd["gu_w"][e], wd["gu_sf"][e], recv_x[d][row], ws2_rows=wd["gu_ws2"][e])
            a = np.array([O.silu(float(v)) for v in h[:I]], np.float32) * h[I:]
            out[d][row] = O.matvec(wd["dn_w"][e], wd["dn_sf"][e], a, ws2_rows=wd["dn_ws2"][e])
    ys = []
    for r in range(world):
        ids, tw = routes[r]
        y = np.zeros((T, H), np.float32)
        for t in range(T):
            for j in range(k):
                d = int(ids[t, j]) // epr
                y[t] += tw[t, j] * out[d][r * R + t * k + j]
        ys.append(y)
    return ys


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_layout_matches_oracle(O, world):
    from nvfp4 import synthetic

    wd = synthetic.moe_weights(E, H, I, seed=5)
    x_all = synthetic.bf16_round(synthetic.activations(3 * world, H, seed=6))
    xs = [x_all[3 * r:3 * (r + 1)] for r in range(world)]
    ys = peer_step_model(O, wd, xs, world, K_TOP)
    ref, _, _ = O.moe(x_all, wd, top_k=K_TOP)
    np.testing.assert_allclose(np.concatenate(ys), ref, rtol=1e-5, atol=1e-6)


def test_peer_windows_table_and_layer_arguments():
    """Host side of the peer exchange without a GPU: the ctypes peer table
    carries rank, world, capacity, hidden size, timeout and every window, and
    EPMoELayer refuses bad exchange arguments before touching the device."""
    from nvfp4 import _lib
    from nvfp4.ep import EPMoELayer, PeerWindows

    pw = PeerWindows(2, 4, 64, 2048, [0x1000, 0x2000, 0x3000, 0x4000], [], [], timeout_ms=250)
    p = pw.peers()
    assert (p.rank, p.world, p.max_rows, p.hidden, p.timeout_ms) == (2, 4, 64, 2048, 250)
    assert [p.windows[i] for i in range(4)] == [0x1000, 0x2000, 0x3000, 0x4000]
    assert all(p.windows[i] is None for i in range(4, _lib.EP_MAX_WORLD))
    pw.close()  # owns nothing: no call into the library
    router = torch.zeros((H, E))
    with pytest.raises(ValueError):
        EPMoELayer(None, router, top_k=K_TOP, num_experts=E, backend=object(), exchange="nvshmem")
    with pytest.raises(ValueError):
        EPMoELayer(None, router, top_k=K_TOP, num_experts=E, backend=object(), exchange="p2p")


def _dropped_rank_worker(rank, world, port, ret):
    import datetime
    import sys
    import time
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nvfp4-mojo_b200"))
    sys.path.insert(0, str(root))
    import torch.distributed as dist
    from nvfp4 import synthetic
    from nvfp4.ep import EPMoELayer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    wd = synthetic.moe_weights(E, H, I, seed=5)
    layer = EPMoELayer(None, torch.from_numpy(wd["router"]), top_k=K_TOP, num_experts=E,
                       backend=CpuBackend(wd, rank, world), static=False)
    if rank == 1:
        ret[1] = "left"
        os._exit(0)  # this rank leaves between steps, without a word to the others
    x = torch.from_numpy(synthetic.bf16_round(synthetic.activations(6, H, seed=6)))
    t0 = time.monotonic()
    try:
        layer(x)
        ret[0] = "no error"
    except Exception as e:  # the exchange with the missing rank must fail, not hang
        ret[0] = type(e).__name__
    ret["t"] = time.monotonic() - t0
    os._exit(0)


def test_dropped_rank_fails_the_exchange_in_bounded_time():
    """A rank that leaves between steps: the surviving rank's next exchange
    (the counts all-to-all) ends with an error within the process group's
    5 s timeout instead of waiting forever."""
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    ret = mgr.dict()
    port = _port()
    procs = [ctx.Process(target=_dropped_rank_worker, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    assert ret.get(1) == "left"
    assert ret.get(0) not in (None, "no error"), ret.get(0)
    assert ret["t"] < 60
