"""The safetensors loader into device memory (include/nvfp4_loader.h): staged
host -> device reads, NVFP4 linears run through the GEMM path, and a MoE
layer (routed experts, shared expert, BF16 router) loaded from the
reference's per-expert tensor layout and run against the oracle."""
import time

import numpy as np
import pytest
import torch

import st_fixtures as F

pytestmark = pytest.mark.gpu


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.sqrt(np.mean(ref * ref)))


def test_read_device_multi_chunk(tmp_path, cuda):
    """A 20 MB tensor crosses the 8 MB staging buffers three times."""
    from nvfp4 import weight_loader as W

    rng = np.random.default_rng(1)
    big = rng.integers(0, 256, size=20 * 1024 * 1024 + 13, dtype=np.uint8)
    F.save(tmp_path / "model.safetensors",
           {"big": torch.from_numpy(big), "small": torch.arange(5, dtype=torch.int32)})
    sf = W.open_safetensors(str(tmp_path / "model.safetensors"))
    dst = torch.empty(big.size, dtype=torch.uint8, device="cuda")
    t0 = time.perf_counter()
    assert sf.read_tensor_into(sf.find_tensor("big"), dst) == big.size
    dt = time.perf_counter() - t0
    assert np.array_equal(dst.cpu().numpy(), big)
    small = torch.empty(5, dtype=torch.int32, device="cuda")
    sf.read_tensor_into(sf.find_tensor("small"), small)
    assert small.cpu().tolist() == [0, 1, 2, 3, 4]
    print(f"file -> device: {big.size / dt / 1e9:.2f} GB/s (page cache)")
    sf.close()


@pytest.mark.parametrize("per_row", [False, True])
def test_load_linear_and_run(O, tmp_path, cuda, per_row):
    import nvfp4
    from nvfp4 import weight_loader as W

    rng = np.random.default_rng(2)
    N, K, M = 512, 1024, 4
    w, sf = F.rand_linear(rng, N, K)
    ws2 = rng.uniform(1e-3, 1e-2, N).astype(np.float32) if per_row else np.float32(3e-3)
    ins = np.float32(0.75)
    t = {}
    F.nvfp4_linear(t, "model.layers.0.self_attn.o_proj", w, sf, ws2=ws2, ins=ins)
    F.save(tmp_path / "model.safetensors", t)
    lw = W.load_linear_safetensors(W.open_model_shards(str(tmp_path)),
                                   "model.layers.0.self_attn.o_proj")
    assert np.array_equal(lw.packed_weights.cpu().numpy(), w)
    assert np.array_equal(lw.blockscales.cpu().numpy(), sf)
    assert lw.input_scale == ins
    if per_row:
        assert np.array_equal(lw.weight_scale_2_rows.cpu().numpy(), ws2)
    else:
        assert lw.weight_scale_2_rows is None and lw.weight_scale_2 == ws2
    x = (rng.standard_normal((M, K))).astype(np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    y = nvfp4.nvfp4_linear(lw.to_linear(), lw.packed_weights, lw.blockscales, xb.cuda(),
                           out_dtype=torch.float32)
    ref = O.linear(w, sf, xb.float().numpy(), input_scale=float(ins),
                   ws2_rows=ws2 if per_row else None, ws2=1.0 if per_row else float(ws2))
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5


def moe_checkpoint(path, E, H, I, Is, seed):
    """A layer in the reference's layout: per-expert gate_proj / up_proj /
    down_proj linears with their own input scales, a shared expert and the
    BF16 router `mlp.gate.weight` [E, H]."""
    from nvfp4 import synthetic

    rng = np.random.default_rng(seed)
    wd = synthetic.moe_weights(E, H, I, seed=seed)
    sd = synthetic.moe_weights(1, H, Is, seed=seed + 1)
    ins = rng.uniform(0.5, 2.0, (E + 1, 3)).astype(np.float32)
    lp = "model.layers.0"
    t = {}

    def put(prefix, w, sf, ws2_rows, s):
        F.nvfp4_linear(t, prefix, w, sf, ws2=ws2_rows, ins=s)

    for e in range(E + 1):
        src, j = (wd, e) if e < E else (sd, 0)
        ii = src["gu_w"].shape[1] // 2
        base = f"{lp}.mlp.experts.{e}" if e < E else f"{lp}.mlp.shared_expert"
        put(base + ".gate_proj", src["gu_w"][j, :ii], src["gu_sf"][j, :ii], src["gu_ws2"][j, :ii],
            ins[e, 0])
        put(base + ".up_proj", src["gu_w"][j, ii:], src["gu_sf"][j, ii:], src["gu_ws2"][j, ii:],
            ins[e, 1])
        put(base + ".down_proj", src["dn_w"][j], src["dn_sf"][j], src["dn_ws2"][j], ins[e, 2])
    router_bf16 = torch.from_numpy(np.ascontiguousarray(wd["router"].T)).to(torch.bfloat16)
    t[f"{lp}.mlp.gate.weight"] = router_bf16
    F.save(path, t)
    # The oracle's dictionaries: input scales folded into the per-row scales,
    # the router as the BF16 values in fp32 [H, E].
    def folded(src, lo, n):
        d = {k: v.copy() for k, v in src.items()}
        ii = d["gu_w"].shape[1] // 2
        for j in range(n):
            d["gu_ws2"][j, :ii] *= ins[lo + j, 0]
            d["gu_ws2"][j, ii:] *= ins[lo + j, 1]
            d["dn_ws2"][j] *= ins[lo + j, 2]
        return d
    ref_routed = folded(wd, 0, E)
    ref_routed["router"] = router_bf16.float().numpy().T.copy()
    ref_shared = folded(sd, E, 1)
    ref_shared["router"] = np.zeros((H, 1), np.float32)
    return ref_routed, ref_shared


def test_load_moe_layer_and_run(O, tmp_path, cuda):
    from nvfp4 import synthetic
    from nvfp4 import weight_loader as W
    from nvfp4.moe import MoELayer

    E, H, I, Is, T, k = 8, 256, 256, 512, 24, 2
    ref_routed, ref_shared = moe_checkpoint(tmp_path / "model.safetensors", E, H, I, Is, seed=11)
    model = W.open_model_shards(str(tmp_path))
    routed = W.load_moe_experts(model, 0)
    shared = W.load_moe_experts(model, 0, shared=True)
    for key, ten in [("gu_w", routed.gate_up), ("gu_sf", routed.gate_up_scale),
                     ("gu_ws2", routed.gate_up_scale_2), ("dn_w", routed.down),
                     ("dn_sf", routed.down_scale), ("dn_ws2", routed.down_scale_2)]:
        assert np.array_equal(ten.cpu().numpy(), ref_routed[key]), key
    assert np.array_equal(routed.router.cpu().numpy(), ref_routed["router"])
    assert np.array_equal(shared.gate_up.cpu().numpy(), ref_shared["gu_w"])
    assert np.array_equal(shared.down_scale_2.cpu().numpy(), ref_shared["dn_ws2"])
    # A slice of the experts (an expert-parallel rank's share).
    part = W.load_moe_experts(model, "model.layers.0", num_experts=3, first=4)
    assert np.array_equal(part.gate_up.cpu().numpy(), ref_routed["gu_w"][4:7])
    assert np.array_equal(part.router.cpu().numpy(), ref_routed["router"][:, 4:7])

    x = synthetic.bf16_round(synthetic.activations(T, H, seed=12))
    X = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = MoELayer(routed, top_k=k, shared=shared)(
        X, out=torch.empty((T, H), dtype=torch.float32, device="cuda"))
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    MoELayer(routed, top_k=k)(X, topk_ids=ids)
    r, _, _ = O.moe(x, ref_routed, top_k=k, force_ids=ids.cpu().numpy(), n_threads=8)
    s, _, _ = O.moe(x, ref_shared, top_k=1, n_threads=8)
    assert rel_err(y.cpu().numpy(), r + s) <= 1e-3
    model.close()


def test_load_qwen35_layer(tmp_path, cuda):
    """load_qwen35_layer: the reference's tensor names for one layer."""
    from nvfp4 import weight_loader as W

    E, H, I, Is = 4, 256, 128, 256
    moe_checkpoint(tmp_path / "experts.safetensors", E, H, I, Is, seed=21)
    rng = np.random.default_rng(22)
    t = {}
    for p, (n, kk) in {"q_proj": (512, H), "k_proj": (128, H), "v_proj": (128, H),
                       "o_proj": (H, 512)}.items():
        w, sf = F.rand_linear(rng, n, kk)
        F.nvfp4_linear(t, f"model.layers.0.self_attn.{p}", w, sf, ws2=np.float32(1e-3))
    t["model.layers.0.input_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
    t["model.layers.0.post_attention_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
    F.save(tmp_path / "attn.safetensors", t)
    model = W.SafetensorsModel.from_files([str(tmp_path / "attn.safetensors"),
                                           str(tmp_path / "experts.safetensors")])
    layer = W.load_qwen35_layer(model, 0, num_experts=E)
    assert layer.q_proj.out_features == 512 and layer.o_proj.in_features == 512
    assert layer.experts.gate_up.shape == (E, 2 * I, H // 2)
    assert layer.shared_expert.gate_up.shape == (1, 2 * Is, H // 2)
    assert layer.input_layernorm.size == 2 * H
    model.close()
