"""Expert-parallel MoE exchange logic on CPU ranks (torch.distributed gloo,
world size 2): the EPMoELayer host algorithm (route -> dispatch plan ->
count / row / expert-id all-to-all -> local experts -> reverse all-to-all ->
combine in slot order) with a CPU backend whose arithmetic is the oracle's.
The result must equal the single-process oracle MoE on the same tokens."""
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

    def experts(self, rows, local_ids):
        O, wd = self.O, self.wd
        out = np.zeros((rows.shape[0], H), np.float32)
        xs = rows.float().numpy()
        for r, le in enumerate(local_ids.numpy()):
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


def _worker(rank, world, port, ret):
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
                           backend=CpuBackend(wd, rank, world))
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


def test_ep_exchange_matches_single_process_oracle(O):
    from nvfp4 import synthetic

    world = 2
    mgr = mp.Manager()
    ret = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), ret), nprocs=world, join=True)
    wd = synthetic.moe_weights(E, H, I, seed=5)
    x_all = synthetic.bf16_round(synthetic.activations(6 * world, H, seed=6))
    ref, _, _ = O.moe(x_all, wd, top_k=K_TOP)
    got = np.concatenate([np.array(ret[r], np.float32) for r in range(world)])
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
