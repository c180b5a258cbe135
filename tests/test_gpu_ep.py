"""Expert-parallel MoE on 2 and 4 GPUs (NCCL all-to-all over NVLink) against the
single-GPU layer: every row an expert computes is the same arithmetic in
both, and the combine sums in the same slot order, so the outputs must be
bitwise equal.  Both exchange modes; the fixed-capacity one also replayed
from a CUDA graph that holds its NCCL calls.  Skipped on a host with fewer
than the test's world size."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

E, H, I, K_TOP, T_RANK = 16, 256, 128, 4, 40


def _worker(rank, world, port, static, ret):
    import datetime
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nvfp4-mojo_b200"))
    sys.path.insert(0, str(root))
    import torch.distributed as dist
    from nvfp4 import synthetic
    from nvfp4.ep import EPMoELayer
    from nvfp4.moe import MoEWeights

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        wd = synthetic.moe_weights(E, H, I, seed=11)
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        local = MoEWeights.from_dict({k: (v[sl] if k != "router" else v) for k, v in wd.items()})
        x_all = synthetic.bf16_round(synthetic.activations(T_RANK * world, H, seed=12))
        x = torch.from_numpy(x_all[T_RANK * rank:T_RANK * (rank + 1)]).cuda().to(torch.bfloat16)
        layer = EPMoELayer(local, local.router, top_k=K_TOP, num_experts=E, static=static)
        y = layer(x)
        torch.cuda.synchronize()
        ret[rank] = y.view(torch.int16).cpu().numpy().tolist()
        if static:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                yg = layer(x)
            g.replay()
            torch.cuda.synchronize()
            ret[f"graph{rank}"] = bool(torch.equal(yg, y))
            del g
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("static", [False, True])
def test_ep_multi_gpu_equals_single_gpu(cuda, static, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from nvfp4 import synthetic
    from nvfp4.moe import MoELayer, MoEWeights

    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), static, ret), nprocs=world, join=True)
    if static:
        assert all(ret[f"graph{r}"] for r in range(world))
    wd = synthetic.moe_weights(E, H, I, seed=11)
    x_all = synthetic.bf16_round(synthetic.activations(T_RANK * world, H, seed=12))
    layer = MoELayer(MoEWeights.from_dict(wd), top_k=K_TOP)
    ref = layer(torch.from_numpy(x_all).cuda().to(torch.bfloat16)).view(torch.int16).cpu().numpy()
    got = np.concatenate([np.array(ret[r], np.int16) for r in range(world)])
    assert np.array_equal(got, ref)
