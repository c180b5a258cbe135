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
    mgr = mp.Manager()
    ret = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), static, ret), nprocs=world, join=True)
    wd = synthetic.moe_weights(E, H, I, seed=5)
    x_all = synthetic.bf16_round(synthetic.activations(6 * world, H, seed=6))
    ref, _, _ = O.moe(x_all, wd, top_k=K_TOP)
    got = np.concatenate([np.array(ret[r], np.float32) for r in range(world)])
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
