"""Gated DeltaNet decode step on the GPU (include/nvfp4_deltanet.h) against
the restated reference deltanet_forward (oracle, nvfp4/deltanet.mojo:335-546)
on the same inputs: NVFP4 projections there are their dequantized weights
times alpha (exact in fp32), B sequences each with its own state, several
steps so the recurrent state and the conv windows carry over.

Tolerances (max |err| / RMS of the reference, per step): projections on fp32
activations 1e-4 for the outputs (the reference's arithmetic; only the
summation order and the place alpha is applied differ), 1e-3 for the
recurrent state, which carries those fp32 differences of near-cancelling
projection outputs from step to step unnormalised (2.6e-4 seen after two
steps of the default layer); on bf16 activations (the decode GEMV) 2e-2 for
both (bf16 hidden state and gated output)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.sqrt(np.mean(ref * ref)))


def build(O, cfg, seed, bias, same_ins=False):
    """Random NVFP4 projections + fp32 small weights, for the GPU and the oracle."""
    import nvfp4
    from nvfp4 import synthetic
    from nvfp4.deltanet import DeltaNetWeights

    rng = np.random.default_rng(seed)
    d, nvh = cfg.d_model, cfg.num_value_heads
    shapes = {"qkv": (cfg.total_qkv_dim(), d), "z": (cfg.z_dim(), d), "b": (nvh, d),
              "a": (nvh, d), "out": (d, cfg.z_dim())}
    gpu, ref = {}, {}
    for i, (name, (n, k)) in enumerate(shapes.items()):
        wd = synthetic.linear_weights(n, k, seed=seed + 10 * i)
        ins = np.float32(rng.uniform(0.5, 1.5))
        if same_ins and name != "out":
            ins = np.float32(0.875)
        lin = nvfp4.NvFp4Linear(k, n, input_scale=float(ins),
                                weight_scale_2_rows=torch.from_numpy(wd["ws2"]).cuda())
        gpu[name] = (lin, torch.from_numpy(wd["w"]).cuda(), torch.from_numpy(wd["sf"]).cuda())
        alpha = (ins * wd["ws2"]).astype(np.float32)
        ref[name] = O.dequant(wd["w"], wd["sf"]) * alpha[:, None]
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    small = dict(a_log=f(nvh) * 0.5, dt_bias=f(nvh) * 0.5,
                 conv_q=f(cfg.q_dim(), cfg.conv_kernel) * 0.5,
                 conv_k=f(cfg.k_dim(), cfg.conv_kernel) * 0.5,
                 conv_v=f(cfg.v_dim(), cfg.conv_kernel) * 0.5)
    if bias:
        small.update(conv_bias_q=f(cfg.q_dim()) * 0.1, conv_bias_k=f(cfg.k_dim()) * 0.1,
                     conv_bias_v=f(cfg.v_dim()) * 0.1)
    ref.update(small)
    w = DeltaNetWeights(**gpu, **{k: torch.from_numpy(v).cuda() for k, v in small.items()})
    return w, ref


def cfg_dict(cfg):
    return dict(d_model=cfg.d_model, num_key_heads=cfg.num_key_heads,
                num_value_heads=cfg.num_value_heads, key_dim=cfg.key_dim,
                value_dim=cfg.value_dim, conv_kernel=cfg.conv_kernel, rms_eps=cfg.rms_eps)


def run_steps(O, cfg, B, steps, proj, tol, seed, bias, tol_state=None, fused=False):
    tol_state = tol if tol_state is None else tol_state
    from nvfp4.deltanet import DeltaNetState, deltanet_forward, fuse_in_proj

    w, ref = build(O, cfg, seed, bias, same_ins=fused)
    if fused:
        w = fuse_in_proj(w)
    state = DeltaNetState(cfg, batch=B)
    ref_states = [O.deltanet_state(cfg_dict(cfg)) for _ in range(B)]
    rng = np.random.default_rng(seed + 99)
    for step in range(steps):
        h = torch.from_numpy(rng.standard_normal((B, cfg.d_model)).astype(np.float32))
        hb = h.to(torch.bfloat16)
        out = torch.empty((B, cfg.d_model), dtype=torch.float32, device="cuda")
        deltanet_forward(hb.cuda(), out, w, state, cfg, proj_dtype=proj)
        got = out.cpu().numpy()
        for b in range(B):
            r = O.deltanet_forward(cfg_dict(cfg), hb[b].float().numpy(), ref, ref_states[b])
            assert rel_err(got[b], r) <= tol, (step, b, rel_err(got[b], r))
    s = state.s_matrix.cpu().numpy()
    for b in range(B):
        assert rel_err(s[b], ref_states[b]["s"]) <= tol_state
        assert rel_err(state.conv_buf_v.cpu().numpy()[b], ref_states[b]["v"]) <= tol_state


@pytest.mark.parametrize("proj,tol,tol_state", [(torch.float32, 1e-4, 1e-3),
                                                (torch.bfloat16, 2e-2, 2e-2)])
@pytest.mark.parametrize("fused", [False, True])
def test_deltanet_small(O, cuda, proj, tol, tol_state, fused):
    """d_model 64, 2 key / 4 value heads of 16 x 16, conv kernel 4 with
    biases, 3 sequences, 3 steps; four input projections or one fused."""
    from nvfp4.deltanet import DeltaNetConfig

    cfg = DeltaNetConfig(d_model=64, num_key_heads=2, num_value_heads=4, key_dim=16,
                         value_dim=16, conv_kernel=4)
    run_steps(O, cfg, B=3, steps=3, proj=proj, tol=tol, seed=5, bias=True, tol_state=tol_state,
              fused=fused)


def test_deltanet_split_heads(O, cuda):
    """value_dim 64 (each head's columns over a cluster of 2 CTAs), key_dim
    48, conv kernel 3, 5 sequences, 3 steps, fp32 projections."""
    from nvfp4.deltanet import DeltaNetConfig

    cfg = DeltaNetConfig(d_model=128, num_key_heads=2, num_value_heads=4, key_dim=48,
                         value_dim=64, conv_kernel=3)
    run_steps(O, cfg, B=5, steps=3, proj=torch.float32, tol=1e-4, seed=9, bias=False,
              tol_state=1e-3)


@pytest.mark.parametrize("proj,tol,tol_state", [(torch.float32, 1e-4, 1e-3),
                                                (torch.bfloat16, 2e-2, 2e-2)])
@pytest.mark.parametrize("fused", [False, True])
def test_deltanet_default_layer(O, cuda, proj, tol, tol_state, fused):
    """The reference's default layer (d_model 2048, 16 key / 32 value heads of
    128 x 128 -- each head over a cluster of 4 CTAs --, conv kernel 4, no
    biases), 2 sequences, 2 steps."""
    from nvfp4.deltanet import DeltaNetConfig

    run_steps(O, DeltaNetConfig(), B=2, steps=2, proj=proj, tol=tol, seed=7, bias=False,
              tol_state=tol_state, fused=fused)


def test_deltanet_validation(cuda):
    import ctypes

    from nvfp4 import _lib
    from nvfp4.deltanet import DeltaNetConfig

    L = _lib.load()
    bad = DeltaNetConfig(value_dim=96).desc()  # not a power of two
    assert L.nvfp4_deltanet_workspace_size(ctypes.byref(bad), 1) == 0
    good = DeltaNetConfig().desc()
    assert L.nvfp4_deltanet_workspace_size(ctypes.byref(good), 4) > 0
