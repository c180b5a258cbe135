"""GPU parity of the NVFP4 MoE layer (router, top-k, grouped gate_up with
SiLU*up, grouped down, combine) against the CPU oracle, through the C ABI.

Tolerances.  fp32 output: max|err| <= 1e-3 * RMS(ref) -- the SiLU*up
activations feed the down projection as bf16 hi + lo parts, so only
summation order and the 2^-16 split residue remain.  bf16 output: per element
|err| <= 2e-2 * RMS(ref) + 2^-8 * |ref|, the bf16-operand bound plus the
output's own rounding (half an ulp of bf16 is up to 2^-8 of the value, and
these synthetic layers have max|y| / RMS(y) up to ~9).
Router near-ties: where two of the oracle's k+1 largest probabilities differ
by less than 1e-5 (at the k-th/(k+1)-th boundary the selection, inside the
top k the order), summation-order differences may legitimately swap them;
such tokens replay the GPU's choice in the oracle (force_ids) and are
counted.  Every other token must select exactly the oracle's experts in the
oracle's order.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2
TIE_GAP = 1e-5


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.sqrt(np.mean(ref * ref)))


def near_ties(probs, k):
    """Tokens whose top-k selection or order is within TIE_GAP of a swap."""
    s = -np.sort(-probs, axis=1)[:, : k + 1]
    return (s[:, :-1] - s[:, 1:]).min(axis=1) < TIE_GAP


def setup(E, H, I, T, seed):
    from nvfp4 import synthetic
    from nvfp4.moe import MoEWeights

    wd = synthetic.moe_weights(E, H, I, seed=seed)
    x = synthetic.bf16_round(synthetic.activations(T, H, seed=seed + 1))
    w = MoEWeights.from_dict(wd)
    return wd, x, w


def check_layer(O, wd, x, w, k, tokens=None, residual=None):
    from nvfp4.moe import MoELayer

    T, H = x.shape
    layer = MoELayer(w, top_k=k)
    X = torch.from_numpy(x).cuda().to(torch.bfloat16)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    tw = torch.empty((T, k), dtype=torch.float32, device="cuda")
    Rz = None if residual is None else torch.from_numpy(residual).cuda().to(torch.bfloat16)
    y = layer(X, residual=Rz, topk_ids=ids, topk_w=tw).float().cpu().numpy()
    y32 = layer(X, residual=Rz, out=torch.empty((T, H), dtype=torch.float32, device="cuda"))
    y32 = y32.cpu().numpy()
    ids = ids.cpu().numpy()
    tok = np.arange(T) if tokens is None else np.asarray(tokens)
    _, probs = O.router(x[tok], wd["router"])
    ties = near_ties(probs, k)
    ref, ref_ids, _ = O.moe(x, wd, top_k=k, tokens=tok, n_threads=8)
    mismatch = [i for i in range(len(tok)) if not np.array_equal(ref_ids[i], ids[tok[i]])]
    assert all(ties[i] for i in mismatch), f"routing differs away from near-ties: {mismatch[:5]}"
    if mismatch:
        ref, _, _ = O.moe(x, wd, top_k=k, tokens=tok, force_ids=ids[tok], n_threads=8)
    if residual is not None:
        ref = ref + residual[tok]
    rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    excess = np.abs(y[tok] - ref) - (TOL * rms + 2.0 ** -8 * np.abs(ref))
    err = rel_err(y[tok], ref)
    assert excess.max() <= 0.0, (err, len(mismatch))
    err32 = rel_err(y32[tok], ref)
    assert err32 <= 1e-3, (err32, len(mismatch))
    return err, len(mismatch)


@pytest.mark.parametrize("T", [1, 5, 64, 300])
def test_moe_small(O, cuda, T):
    wd, x, w = setup(E=8, H=256, I=128, T=T, seed=T)
    check_layer(O, wd, x, w, k=2)


@pytest.mark.parametrize("T", [1, 16, 256])
def test_moe_config3(O, cuda, T):
    """One MoE FFN layer: 128 experts, top-8, hidden 2048, intermediate 768."""
    wd, x, w = setup(E=128, H=2048, I=768, T=T, seed=100 + T)
    check_layer(O, wd, x, w, k=8)


@pytest.mark.parametrize("E,H,I,T", [(8, 512, 3072, 5), (4, 6144, 256, 3)])
def test_moe_clustered_expert_gemv_fallback(O, cuda, E, H, I, T):
    """Shapes whose work-item activations do not fit beside a two-stage ring
    in one CTA's shared memory: the down GEMV (I = 3072) or the gate_up GEMV
    (H = 6144) runs as one cluster grid per item instead of the persistent
    grouped kernel; the other GEMV of the layer stays persistent."""
    wd, x, w = setup(E=E, H=H, I=I, T=T, seed=400 + T)
    check_layer(O, wd, x, w, k=2)


def test_moe_config3_large_sampled(O, cuda):
    """T = 4096 tokens, oracle on a sample of tokens; with a residual add."""
    T = 4096
    wd, x, w = setup(E=128, H=2048, I=768, T=T, seed=7)
    res = np.random.default_rng(8).standard_normal((T, 2048)).astype(np.float32)
    res = torch.from_numpy(res).to(torch.bfloat16).float().numpy()
    tok = np.sort(np.random.default_rng(9).choice(T, 48, replace=False))
    check_layer(O, wd, x, w, k=8, tokens=tok, residual=res)


def test_route_matches_oracle(O, cuda):
    from nvfp4.moe import moe_route

    wd, x, w = setup(E=128, H=2048, I=768, T=512, seed=3)
    ids, tw, logits = moe_route(w, torch.from_numpy(x).cuda().to(torch.bfloat16), top_k=8)
    ref_logits, probs = O.router(x, wd["router"])
    assert rel_err(logits.cpu().numpy(), ref_logits) <= 1e-5
    ids = ids.cpu().numpy()
    ties = near_ties(probs, 8)
    for t in range(x.shape[0]):
        order = sorted(range(128), key=lambda e: (-probs[t, e], e))[:8]
        if not ties[t]:
            assert list(ids[t]) == order
    s = tw.cpu().numpy().sum(1)
    assert np.allclose(s, 1.0, atol=1e-5)


def test_experts_rows_and_invalid_ids(O, cuda):
    """moe_experts over explicit rows; rows with expert id -1 stay untouched."""
    from nvfp4.moe import moe_experts

    E, H, I, R = 16, 256, 128, 40
    wd, x, w = setup(E=E, H=H, I=I, T=R, seed=21)
    rng = np.random.default_rng(22)
    ids = rng.integers(0, E, R).astype(np.int32)
    ids[[3, 17]] = -1
    out = torch.full((R, H), 7.0, dtype=torch.float32, device="cuda")
    moe_experts(w, torch.from_numpy(x).cuda().to(torch.bfloat16),
                torch.from_numpy(ids).cuda(), out=out, top_k=2)
    got = out.float().cpu().numpy()
    assert np.all(got[[3, 17]] == 7.0)
    for r in range(R):
        if ids[r] < 0:
            continue
        e = ids[r]
        h = O.matvec(wd["gu_w"][e], wd["gu_sf"][e], x[r], ws2_rows=wd["gu_ws2"][e])
        a = np.array([O.silu(float(v)) for v in h[:I]], np.float32) * h[I:]
        y = O.matvec(wd["dn_w"][e], wd["dn_sf"][e], a, ws2_rows=wd["dn_ws2"][e])
        assert rel_err(got[r], y) <= TOL, r


@pytest.mark.parametrize("E,H,I", [(16, 512, 256), (128, 2048, 768)])
def test_experts_gemv_path_repeated(O, cuda, E, H, I):
    """Expert GEMMs on the decode GEMV path (shapes with H, I % 256 == 0 and
    few rows per expert): one expert with 3 full items of 8 rows, others with
    1-2 rows, rows with expert id -1; called twice in a row on fresh inputs
    with the same workspace (the second call must not see the first's
    data).  fp32 rows within 1e-3 RMS of the oracle's expert chain."""
    from nvfp4.moe import moe_experts

    R = 64
    wd, _, w = setup(E=E, H=H, I=I, T=1, seed=31)
    rng = np.random.default_rng(32)
    ws = torch.empty(1 << 26, dtype=torch.uint8, device="cuda")
    for call in range(2):
        x = synthetic_x(R, H, seed=40 + call, scale=1 + 5 * call)
        ids = rng.integers(0, E, R).astype(np.int32)
        ids[:24] = 3
        ids[[30, 41]] = -1
        out = torch.full((R, H), 7.0, dtype=torch.float32, device="cuda")
        moe_experts(w, torch.from_numpy(x).cuda().to(torch.bfloat16),
                    torch.from_numpy(ids).cuda(), out=out, top_k=2, workspace=ws)
        got = out.cpu().numpy()
        assert np.all(got[[30, 41]] == 7.0)
        for r in range(R):
            if ids[r] < 0:
                continue
            e = ids[r]
            h = O.matvec(wd["gu_w"][e], wd["gu_sf"][e], x[r], ws2_rows=wd["gu_ws2"][e])
            a = np.array([O.silu(float(v)) for v in h[:I]], np.float32) * h[I:]
            y = O.matvec(wd["dn_w"][e], wd["dn_sf"][e], a, ws2_rows=wd["dn_ws2"][e])
            assert rel_err(got[r], y) <= 1e-3, (call, r)


def synthetic_x(R, H, seed, scale=1.0):
    from nvfp4 import synthetic

    return synthetic.bf16_round(synthetic.activations(R, H, seed=seed) * scale)


def test_workspace_too_small_is_an_error(cuda):
    import ctypes

    from nvfp4 import _lib
    from nvfp4.moe import MoELayer

    _, x, w = setup(E=8, H=256, I=128, T=4, seed=1)
    layer = MoELayer(w, top_k=2)
    X = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = torch.empty_like(X)
    ws = torch.empty(64, dtype=torch.uint8, device="cuda")
    rc = _lib.load().nvfp4_moe_forward(ctypes.byref(layer.desc), ctypes.byref(layer.ptrs),
                                        X.data_ptr(), None, y.data_ptr(), _lib.DTYPE_BF16, 4,
                                        None, None,
                                        ws.data_ptr(), ws.numel(), None)
    assert rc == _lib.NVFP4_ERR_WORKSPACE


def test_moe_tensor_core_path_small(O, cuda):
    """Many rows per expert (R >= 64 E) with H, I multiples of 256: the grouped
    tcgen05 GEMMs (gate_up with two accumulators and fused SiLU*up, down on the
    hi + lo activation parts), items of up to 128 rows, ragged last items."""
    wd, x, w = setup(E=8, H=512, I=256, T=400, seed=31)
    check_layer(O, wd, x, w, k=2)


def test_moe_tensor_core_path_config3(O, cuda):
    """Config-3 layer at T = 1024 (R = 8192 = 64 E: tensor-core path), sampled."""
    T = 1024
    wd, x, w = setup(E=128, H=2048, I=768, T=T, seed=33)
    tok = np.sort(np.random.default_rng(34).choice(T, 64, replace=False))
    check_layer(O, wd, x, w, k=8, tokens=tok)


def shared_expert_dict(H, Is, seed):
    """A one-expert stack whose zero router [H, 1] gives every token weight 1:
    the oracle's MoE layer over it is the shared expert alone."""
    from nvfp4 import synthetic

    sd = synthetic.moe_weights(1, H, Is, seed=seed)
    sd["router"] = np.zeros((H, 1), np.float32)
    return sd


@pytest.mark.parametrize("T,E,H,I,Is,k", [(1, 16, 512, 256, 512, 4),
                                          (16, 128, 2048, 768, 1024, 8),
                                          (40, 16, 512, 256, 512, 4),
                                          (300, 16, 512, 256, 768, 4)])
def test_moe_shared_expert(O, cuda, T, E, H, I, Is, k):
    """Routed experts plus the always-on shared expert (weight 1), with a
    residual: the shared expert's rows take the GEMV (T <= 32), skinny (T = 40)
    and tensor-core (T = 300) expert paths.  Oracle: the routed layer plus the
    shared expert as a one-expert layer, summed in fp32 in that order."""
    from nvfp4.moe import MoELayer, MoEWeights

    wd, x, w = setup(E=E, H=H, I=I, T=T, seed=50 + T)
    sd = shared_expert_dict(H, Is, seed=60 + T)
    shared = MoEWeights.from_dict({kk: v for kk, v in sd.items() if kk != "router"})
    res = synthetic_x(T, H, seed=70 + T)
    layer = MoELayer(w, top_k=k, shared=shared)
    X = torch.from_numpy(x).cuda().to(torch.bfloat16)
    Rz = torch.from_numpy(res).cuda().to(torch.bfloat16)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    y = layer(X, residual=Rz, topk_ids=ids).float().cpu().numpy()
    y32 = layer(X, residual=Rz, out=torch.empty((T, H), dtype=torch.float32, device="cuda"))
    y32 = y32.cpu().numpy()
    ids = ids.cpu().numpy()
    _, probs = O.router(x, wd["router"])
    ties = near_ties(probs, k)
    routed, ref_ids, _ = O.moe(x, wd, top_k=k, n_threads=8)
    mismatch = [t for t in range(T) if not np.array_equal(ref_ids[t], ids[t])]
    assert all(ties[t] for t in mismatch), mismatch[:5]
    if mismatch:
        routed, _, _ = O.moe(x, wd, top_k=k, force_ids=ids, n_threads=8)
    sh, sh_ids, sh_w = O.moe(x, sd, top_k=1, n_threads=8)
    assert np.all(sh_ids == 0) and np.all(sh_w == 1.0)
    ref = (routed + sh) + res
    rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    assert (np.abs(y - ref) - (TOL * rms + 2.0 ** -8 * np.abs(ref))).max() <= 0.0
    assert rel_err(y32, ref) <= 1e-3
    # The shared expert's contribution is not lost in the residual.
    assert rel_err(y32 - (routed + res), sh) <= 1e-2


def test_stack_gate_up_prepack(O, cuda):
    """Separate per-expert gate_proj / up_proj linears (different input scales,
    one of them a per-tensor weight_scale_2) stacked by nvfp4_stack_rows give
    the stacked layout bit for bit, with the input scales folded into the
    per-row scales; the layer over them matches the oracle."""
    from nvfp4.moe import MoEWeights, stack_gate_up

    E, H, I, T, k = 4, 256, 128, 24, 2
    wd, x, _ = setup(E=E, H=H, I=I, T=T, seed=81)
    rng = np.random.default_rng(82)
    ins = rng.uniform(0.5, 2.0, (E, 2)).astype(np.float32)
    wd["gu_ws2"][2, :I] = wd["gu_ws2"][2, 0]  # expert 2's gate_proj: one scale
    gates, ups = [], []
    for e in range(E):
        g_ws2 = np.float32(wd["gu_ws2"][e, 0]) if e == 2 else torch.from_numpy(wd["gu_ws2"][e, :I])
        gates.append({"w": torch.from_numpy(wd["gu_w"][e, :I]).cuda(),
                      "sf": torch.from_numpy(wd["gu_sf"][e, :I]),
                      "ws2": g_ws2, "in": ins[e, 0]})
        ups.append({"w": torch.from_numpy(wd["gu_w"][e, I:]),
                    "sf": torch.from_numpy(wd["gu_sf"][e, I:]).cuda(),
                    "ws2": torch.from_numpy(wd["gu_ws2"][e, I:]), "in": ins[e, 1]})
    gw, gsf, gws2 = stack_gate_up(gates, ups)
    torch.cuda.synchronize()
    assert np.array_equal(gw.cpu().numpy(), wd["gu_w"])
    assert np.array_equal(gsf.cpu().numpy(), wd["gu_sf"])
    folded = wd["gu_ws2"] * np.repeat(ins, I, axis=1)
    assert np.array_equal(gws2.cpu().numpy(), folded)
    wd["gu_ws2"] = folded
    w = MoEWeights.from_dict(dict(wd, gu_w=gw, gu_sf=gsf, gu_ws2=gws2))
    check_layer(O, wd, x, w, k=k)


def test_experts_gemv_path_repeatable(cuda):
    """The grouped-GEMV expert path at the config-3 layer with T = 256
    (2048 slots, items of up to 8 slots): 25 calls with the same routing give
    bitwise identical expert outputs, although the slot order inside each
    expert's group (shared-memory atomics) differs from call to call.  Each
    staged weight chunk must be read before TMA refills its buffer; a refill
    that overtook the reads corrupted rows of one item in a few calls of 60."""
    from nvfp4.moe import moe_experts, moe_route

    E, H, I, T, k = 128, 2048, 768, 256, 8
    R = T * k
    wd, x, w = setup(E=E, H=H, I=I, T=T, seed=100 + T)
    X = torch.from_numpy(x).cuda().to(torch.bfloat16)
    ids, _, _ = moe_route(w, X, top_k=k)
    row_expert = ids.reshape(-1).contiguous()
    slot_tok = (torch.arange(R, device="cuda", dtype=torch.int32) // k).contiguous()
    ws = torch.empty(1 << 26, dtype=torch.uint8, device="cuda")
    first = None
    for i in range(25):
        y = torch.full((R, H), float("nan"), dtype=torch.float32, device="cuda")
        moe_experts(w, X, row_expert, x_row_index=slot_tok, out=y, top_k=k, workspace=ws)
        if first is None:
            first = y
            assert not torch.isnan(first).any()
        else:
            assert torch.equal(y, first), f"call {i} differs"
