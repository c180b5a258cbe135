"""Column split of one NVFP4 linear across ranks (nvfp4/column_split.py): the
shard bounds, and the split + all-gather on CPU ranks (gloo, world size 2 and
3, the oracle's linear as each rank's compute) against the single-process
oracle, bit for bit; on 2 GPUs (NCCL) against the single-GPU linear."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

N, K, M = 200, 512, 5  # N not a multiple of the 16-row tile x world


def test_shard_bounds_cover_tiles_evenly():
    from nvfp4.column_split import TILE_ROWS, shard_bounds

    for n in (1, 15, 16, 17, 200, 1536, 14336):
        for world in (1, 2, 3, 4, 8):
            b = [shard_bounds(n, world, r) for r in range(world)]
            assert b[0][0] == 0 and b[-1][1] == n
            for (a0, a1), (c0, c1) in zip(b, b[1:]):
                assert a1 == c0
            for a0, a1 in b:
                assert a0 % TILE_ROWS == 0 and a1 >= a0
            tiles = [(-(-(a1 - a0) // TILE_ROWS)) for a0, a1 in b]
            assert max(tiles) - min(tiles) <= 1
    with pytest.raises(ValueError):
        shard_bounds(16, 2, 2)


def _oracle_compute(linear, w, sf, x, out_dtype=torch.float32, flags=0):
    from oracle import oracle as O

    rows = linear.weight_scale_2_rows
    y = O.linear(w.numpy(), sf.numpy(), x.float().numpy(), input_scale=linear.input_scale,
                 ws2=linear.weight_scale_2, ws2_rows=None if rows is None else rows.numpy())
    return torch.from_numpy(y).to(out_dtype)


def _cpu_worker(rank, world, port, ret):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nvfp4-mojo_b200"))
    sys.path.insert(0, str(root))
    import torch.distributed as dist
    from nvfp4 import NvFp4Linear, synthetic
    from nvfp4.column_split import ColumnSplitLinear

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wd = synthetic.linear_weights(N, K, seed=3)
        x = torch.from_numpy(synthetic.bf16_round(synthetic.activations(M, K, seed=4)))
        lin = NvFp4Linear(K, N, input_scale=0.5, weight_scale_2_rows=torch.from_numpy(wd["ws2"]))
        split = ColumnSplitLinear(lin, torch.from_numpy(wd["w"]), torch.from_numpy(wd["sf"]),
                                  compute=_oracle_compute)
        ret[f"slice{rank}"] = (split.n0, split.n1, split(x, out_dtype=torch.float32).tolist())
        ret[rank] = split(x, out_dtype=torch.float32, gather=True).tolist()
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 3])
def test_column_split_on_cpu_ranks_equals_oracle(O, world):
    from nvfp4 import synthetic

    ret = mp.get_context("spawn").Manager().dict()
    mp.spawn(_cpu_worker, args=(world, _port(), ret), nprocs=world, join=True)
    wd = synthetic.linear_weights(N, K, seed=3)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=4))
    ref = O.linear(wd["w"], wd["sf"], x, input_scale=0.5, ws2_rows=wd["ws2"])
    for r in range(world):
        n0, n1, ys = ret[f"slice{r}"]
        assert np.array_equal(np.array(ys, np.float32), ref[:, n0:n1])
        assert np.array_equal(np.array(ret[r], np.float32), ref)


def _gpu_worker(rank, world, port, ret):
    import datetime
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nvfp4-mojo_b200"))
    sys.path.insert(0, str(root))
    import torch.distributed as dist
    from nvfp4 import NvFp4Linear, synthetic
    from nvfp4.column_split import ColumnSplitLinear

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        n, k = 1536, 2048
        wd = synthetic.linear_weights(n, k, seed=7)
        lin = NvFp4Linear(k, n, weight_scale_2_rows=torch.from_numpy(wd["ws2"]).to(dev))
        split = ColumnSplitLinear(lin, torch.from_numpy(wd["w"]).to(dev),
                                  torch.from_numpy(wd["sf"]).to(dev))
        out = {}
        for m in (1, 8, 64):
            x = torch.from_numpy(synthetic.bf16_round(synthetic.activations(m, k, seed=8 + m)))
            y = split(x.to(dev, torch.bfloat16), out_dtype=torch.float32, gather=True)
            out[m] = y.cpu().numpy().tolist()
        ret[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_column_split_two_gpus_equals_single_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from nvfp4 import NvFp4Linear, nvfp4_linear, synthetic

    ret = mp.get_context("spawn").Manager().dict()
    mp.spawn(_gpu_worker, args=(2, _port(), ret), nprocs=2, join=True)
    n, k = 1536, 2048
    wd = synthetic.linear_weights(n, k, seed=7)
    lin = NvFp4Linear(k, n, weight_scale_2_rows=torch.from_numpy(wd["ws2"]).cuda())
    w, sf = torch.from_numpy(wd["w"]).cuda(), torch.from_numpy(wd["sf"]).cuda()
    for m in (1, 8, 64):
        x = torch.from_numpy(synthetic.bf16_round(synthetic.activations(m, k, seed=8 + m)))
        ref = nvfp4_linear(lin, w, sf, x.cuda().to(torch.bfloat16),
                           out_dtype=torch.float32).cpu().numpy()
        rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
        for r in range(2):
            y = np.array(ret[r][m], np.float32)
            # Each rank's kernel plan follows its slice's shape (K split), so
            # fp32 sums may differ in order from the whole-matrix launch.
            assert np.max(np.abs(y - ref)) <= 1e-5 * rms, (r, m)
