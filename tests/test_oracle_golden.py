"""Pins the CPU oracle (and the host-side config mirror) to the reference's own
known-answer tests and to independent implementations.  CPU only."""
import json
import math
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"
KATS = json.loads((GOLD / "reference_kats.json").read_text())
TOL = KATS["tolerance"]["abs_or_rel"]  # tests/helpers.mojo:4-28


def approx_eq(a, b, tol=TOL):
    """tests/helpers.mojo:4-16: absolute, else relative to max(a, b)."""
    d = abs(a - b)
    if d <= tol:
        return True
    den = abs(a if a > b else b)
    return den > 0 and d / den <= tol


def test_lut_matches_reference_kat(O):
    import nvfp4

    for i, v in enumerate(KATS["lut"]["values"]):
        exp = float(v)
        assert approx_eq(O.lut(i), exp)
        assert approx_eq(nvfp4.FP4_E2M1_LUT[i], exp)
        # code 8 is -0.0: sign must survive (the KAT writes "-0.0").
        assert math.copysign(1.0, O.lut(i)) == math.copysign(1.0, exp)
        assert math.copysign(1.0, nvfp4.FP4_E2M1_LUT[i]) == math.copysign(1.0, exp)


def test_pack_unpack_kat(O):
    import nvfp4

    k = KATS["pack_unpack"]
    assert O.pack_fp4_pair(k["lo"], k["hi"]) == k["packed"]
    assert O.unpack_fp4_pair(k["packed"]) == (k["lo"], k["hi"])
    assert nvfp4.pack_fp4_pair(k["lo"], k["hi"]) == k["packed"]
    assert nvfp4.unpack_fp4_pair(k["packed"]) == (k["lo"], k["hi"])
    for b in range(256):  # round trip over every byte
        lo, hi = O.unpack_fp4_pair(b)
        assert O.pack_fp4_pair(lo, hi) == b
        assert nvfp4.pack_fp4_pair(*nvfp4.unpack_fp4_pair(b)) == b


def test_dequant_kat(O):
    import nvfp4

    cases = KATS["dequant"]["cases"]
    assert len(cases) == 7
    for c in cases:
        assert approx_eq(O.dequant_fp4(c["code"], c["scale"]), c["expected"])
        assert approx_eq(nvfp4.dequant_fp4(c["code"], c["scale"]), c["expected"])


def test_config_kat():
    import torch
    import nvfp4

    k = KATS["config"]
    cfg = nvfp4.NvFp4Config()
    assert nvfp4.NVFP4_PACK_FACTOR == k["pack_factor"]
    assert cfg.group_size == nvfp4.NVFP4_GROUP_SIZE == k["group_size"]
    assert cfg.weight_dtype == getattr(torch, k["weight_dtype"])
    assert cfg.scale_dtype == getattr(torch, k["scale_dtype"].replace("float8_e4m3fn", "float8_e4m3fn"))
    assert cfg.output_dtype == getattr(torch, k["output_dtype"])
    lin = nvfp4.NvFp4Linear(2048, 1536)
    assert lin.input_scale == 1.0 and lin.weight_scale_2 == 1.0  # config.mojo:78-79
    assert lin.packed_weight_size() == 1536 * 1024
    assert lin.scale_size() == 1536 * 128


def test_activation_kats(O):
    import nvfp4

    for fn in ("sigmoid", "silu"):
        for c in KATS["activations"][fn]:
            assert approx_eq(getattr(O, fn)(c["x"]), c["expected"]), (fn, c)
            assert approx_eq(getattr(nvfp4, fn)(c["x"]), c["expected"]), (fn, c)


def test_e4m3_decode_matches_ml_dtypes_table(O):
    ref = json.loads((GOLD / "e4m3_table.json").read_text())["values"]
    ours = O.e4m3_table()
    for b in range(256):
        r = ref[b]
        if r == "nan":
            assert math.isnan(ours[b]), b
            assert b in (0x7F, 0xFF)
        else:
            assert ours[b] == float(r), (b, ours[b], r)
            assert math.copysign(1.0, ours[b]) == math.copysign(1.0, float(r))


def test_e4m3_encode_round_trip_and_rne(O):
    tab = O.e4m3_table()
    for b in range(256):
        if b in (0x7F, 0xFF):
            continue
        assert O.f32_to_e4m3(float(tab[b])) in (b, b ^ 0x80 if tab[b] == 0 else b)
    # torch's float8_e4m3fn cast is an independent RNE implementation.
    import torch

    xs = np.random.default_rng(7).uniform(-500, 500, 4000).astype(np.float32)
    xs = np.concatenate([xs, np.float32([0.0009765625, 0.0029296875, 1.0625, 17.0, 450.0])])
    mine = np.array([O.f32_to_e4m3(float(x)) for x in xs], dtype=np.uint8)
    theirs = torch.from_numpy(np.clip(xs, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, theirs)


def test_e2m1_encode_rne(O):
    # Midpoints round to the even code; values past 6 saturate.
    cases = {0.25: 0, 0.75: 2, 1.25: 2, 1.75: 4, 2.5: 4, 3.5: 6, 5.0: 6, 7.0: 7, 100.0: 7,
             0.3: 1, 2.9: 5, -0.75: 10, -6.5: 15}
    for x, code in cases.items():
        assert O.f32_to_e2m1(x) == code, (x, O.f32_to_e2m1(x), code)
    for c in range(16):
        assert O.f32_to_e2m1(O.lut(c)) == c


def _numpy_dequant(w, sf, tab):
    lut = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float64)
    lo, hi = w & 15, w >> 4
    codes = np.stack([lo, hi], axis=-1).reshape(w.shape[0], -1)
    scale = np.repeat(tab[sf].astype(np.float64), 16, axis=1)
    return lut[codes] * scale


def test_oracle_dequant_and_matvec_vs_numpy(O):
    from nvfp4 import synthetic

    N, K, M = 1536, 2048, 4
    wd = synthetic.linear_weights(N, K, seed=0)
    x = synthetic.activations(M, K, seed=1)
    tab = O.e4m3_table()
    deq = _numpy_dequant(wd["w"], wd["sf"], tab)
    assert np.array_equal(O.dequant(wd["w"], wd["sf"]), deq.astype(np.float32))
    # Sub-tile with offsets (reference tile form).
    t = O.dequant_tile(wd["w"], wd["sf"], K // 2, K // 16, 5, 48, 7, 64)
    assert np.array_equal(t, deq[5:12, 48:112].astype(np.float32))
    # Independent float64 evaluation vs the fp32 sequential loop.
    ref64 = (x.astype(np.float64) @ deq.T) * (1.0 * wd["ws2"][None, :].astype(np.float64))
    y = O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"])
    err = np.abs(y - ref64).max()
    bound = 4e-7 * K * np.abs(x).max() * np.abs(deq).max() * wd["ws2"].max()
    assert err <= bound, (err, bound)
    # matvec (scalar ws2 = reference form) agrees with linear row by row.
    y0 = O.matvec(wd["w"], wd["sf"], x[0], input_scale=0.5, ws2=0.25)
    y1 = O.linear(wd["w"], wd["sf"], x[:1], input_scale=0.5, ws2=0.25)[0]
    assert np.array_equal(y0, y1)


def test_oracle_gemm_kernel_layout(O):
    from nvfp4 import synthetic

    N, K, M = 64, 256, 5
    wd = synthetic.linear_weights(N, K, seed=3)
    x = synthetic.activations(M, K, seed=4)
    out = O.gemm_kernel(wd["w"], wd["sf"], np.ascontiguousarray(x.T), alpha=0.75)
    ref = O.linear(wd["w"], wd["sf"], x, input_scale=0.75, ws2=1.0)
    assert np.array_equal(out, ref.T)


def test_oracle_sampled_linear(O):
    from nvfp4 import synthetic

    N, K, M = 96, 512, 9
    wd = synthetic.linear_weights(N, K, seed=5)
    x = synthetic.activations(M, K, seed=6)
    full = O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"])
    rows, cols = np.array([0, 4, 8]), np.array([1, 50, 95])
    part = O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"], rows=rows, cols=cols, n_threads=2)
    assert np.array_equal(part, full[np.ix_(rows, cols)])


def test_oracle_quantize_act_properties(O):
    x = np.random.default_rng(9).standard_normal((3, 64)).astype(np.float32)
    ins = float(np.abs(x).max() / (6 * 448))
    q, s = O.quantize_act(x, ins)
    tab = O.e4m3_table()
    deq = _numpy_dequant(q, s, tab) * ins
    # NVFP4 round trip: error at most half an E2M1 step of the block scale.
    blk = np.abs(x).reshape(3, 4, 16).max(-1)
    step = np.repeat(blk / 6.0 * 2.0, 16, axis=1).reshape(3, 64)  # <= 1 ulp at 6 (spacing 2)
    assert np.all(np.abs(deq - x) <= step * 0.5 + 1e-6)


def test_oracle_router_and_moe_small(O):
    from nvfp4 import synthetic

    E, H, I, T, k = 8, 64, 32, 5, 2
    w = synthetic.moe_weights(E, H, I, seed=11)
    x = synthetic.activations(T, H, seed=12)
    logits, probs = O.router(x, w["router"])
    assert np.allclose(probs.sum(1), 1.0, atol=1e-6)
    out, ids, tw = O.moe(x, w, top_k=k)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-probs[t, e], e))[:k]
        assert list(ids[t]) == order
        assert np.isclose(tw[t].sum(), 1.0, atol=1e-6)
    # Recompute one token with the matvec building blocks.
    t = 2
    ref = np.zeros(H, np.float32)
    for j in range(k):
        e = ids[t, j]
        h = O.matvec(w["gu_w"][e], w["gu_sf"][e], x[t], ws2_rows=w["gu_ws2"][e])
        a = np.array([O.silu(float(v)) for v in h[:I]], np.float32) * h[I:]
        y = O.matvec(w["dn_w"][e], w["dn_sf"][e], a, ws2_rows=w["dn_ws2"][e])
        ref += tw[t, j] * y
    assert np.allclose(out[t], ref, rtol=1e-5, atol=1e-6)
    part, pids, _ = O.moe(x, w, top_k=k, tokens=[4, 1])
    assert np.array_equal(part, out[[4, 1]]) and np.array_equal(pids, ids[[4, 1]])
