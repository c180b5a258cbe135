"""ctypes front-end of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference leg of bench.py, always as the checker or the
timed CPU baseline, never as part of the product path.

Each wrapper names the reference function it restates (see nvfp4_oracle.c).
Arrays are numpy; floats are float32, codes uint8.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def use_native_build() -> str:
    """Switches this process to the timing build of the same C sources,
    compiled for this host (-O3 -march=native, no FMA contraction), building
    it on first use; falls back to the portable build when no compiler is
    present.  Called by the CPU-baseline leg of bench.py only.  Returns a
    description of the build in use."""
    global _lib, _LIB_PATH
    import tempfile

    # A fresh path per process: a build made on another host is never reused.
    native = Path(tempfile.mkdtemp(prefix="oracle-native-")) / "liboracle_native.so"
    try:
        subprocess.run(["make", "-s", "-C", str(_HERE), "native", f"NATIVE_LIB={native}"],
                       check=True, capture_output=True, timeout=120)
    except (OSError, subprocess.SubprocessError):
        return "portable build (-O3, no -march=native): the native build failed on this host"
    _LIB_PATH, _lib = native, None
    lib()
    return "gcc -O3 -march=native -ffp-contract=off -fopenmp, built on this host"


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        L.oracle_lut.restype = ctypes.c_float
        L.oracle_lut.argtypes = [ctypes.c_int]
        L.oracle_dequant_fp4.restype = ctypes.c_float
        L.oracle_dequant_fp4.argtypes = [ctypes.c_uint8, ctypes.c_float]
        L.oracle_pack_fp4_pair.restype = ctypes.c_uint8
        L.oracle_pack_fp4_pair.argtypes = [ctypes.c_uint8, ctypes.c_uint8]
        L.oracle_unpack_fp4_pair.restype = None
        L.oracle_unpack_fp4_pair.argtypes = [ctypes.c_uint8, _u8p, _u8p]
        L.oracle_compute_effective_scale.restype = ctypes.c_float
        L.oracle_compute_effective_scale.argtypes = [ctypes.c_float] * 3
        L.oracle_e4m3_to_f32.restype = ctypes.c_float
        L.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.oracle_f32_to_e4m3_satfinite.restype = ctypes.c_uint8
        L.oracle_f32_to_e4m3_satfinite.argtypes = [ctypes.c_float]
        L.oracle_f32_to_e2m1_satfinite.restype = ctypes.c_uint8
        L.oracle_f32_to_e2m1_satfinite.argtypes = [ctypes.c_float]
        L.oracle_sigmoid.restype = ctypes.c_float
        L.oracle_sigmoid.argtypes = [ctypes.c_float]
        L.oracle_silu.restype = ctypes.c_float
        L.oracle_silu.argtypes = [ctypes.c_float]
        L.oracle_dequant_tile.restype = None
        L.oracle_dequant_tile.argtypes = [_u8p, _u8p, _f32p] + [_i64] * 6
        L.oracle_matvec.restype = None
        L.oracle_matvec.argtypes = [_i64, _i64, ctypes.c_float, ctypes.c_float,
                                    _f32p, _u8p, _u8p, _f32p, _f32p]
        L.oracle_linear.restype = None
        L.oracle_linear.argtypes = [_i64, _i64, _i64, ctypes.c_float, ctypes.c_float,
                                    _f32p, _u8p, _u8p, _f32p, _f32p,
                                    _i64p, _i64, _i64p, _i64, ctypes.c_int]
        L.oracle_gemm_kernel.restype = None
        L.oracle_gemm_kernel.argtypes = [_i64, _i64, _i64, _u8p, _u8p, _f32p, _f32p,
                                         ctypes.c_float]
        L.oracle_quantize_act.restype = None
        L.oracle_quantize_act.argtypes = [_i64, _i64, _f32p, ctypes.c_float, _u8p, _u8p]
        L.oracle_router.restype = None
        L.oracle_router.argtypes = [_i64, _i64, _i64, _f32p, _f32p, _f32p, _f32p]
        L.oracle_moe.restype = None
        L.oracle_moe.argtypes = [_i64, _i64, _i64, _i64, _i64, ctypes.c_int,
                                 _f32p, _f32p, _u8p, _u8p, _f32p, _f32p,
                                 _u8p, _u8p, _f32p, _f32p, _f32p,
                                 _i64p, _i64, _i32p, _f32p, _i32p, ctypes.c_int]
        L.oracle_softplus.restype = ctypes.c_float
        L.oracle_softplus.argtypes = [ctypes.c_float]
        L.oracle_dn_matvec.restype = None
        L.oracle_dn_matvec.argtypes = [_f32p, _f32p, _f32p, _i64, _i64]
        L.oracle_dn_matvec_t.restype = None
        L.oracle_dn_matvec_t.argtypes = [_f32p, _f32p, _f32p, _i64, _i64]
        L.oracle_rms_norm.restype = None
        L.oracle_rms_norm.argtypes = [_f32p, _i64, ctypes.c_float]
        L.oracle_conv1d_step.restype = None
        L.oracle_conv1d_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _f32p]
        L.oracle_deltanet_forward.restype = None
        L.oracle_deltanet_forward.argtypes = ([_i64] * 6 + [ctypes.c_float] + [_f32p] * 2
                                              + [_f32p] * 5 + [_f32p] * 2 + [_f32p] * 6
                                              + [_f32p] * 4)
        _lib = L
    return _lib


def _p(a, t):
    if a is None:
        return ctypes.cast(None, t)
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


def lut(code: int) -> float:
    return lib().oracle_lut(code)


def dequant_fp4(v: int, scale: float) -> float:
    return lib().oracle_dequant_fp4(v, scale)


def pack_fp4_pair(lo: int, hi: int) -> int:
    return lib().oracle_pack_fp4_pair(lo, hi)


def unpack_fp4_pair(b: int):
    lo, hi = ctypes.c_uint8(), ctypes.c_uint8()
    lib().oracle_unpack_fp4_pair(b, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def compute_effective_scale(bs: float, ws2: float, ins: float) -> float:
    return lib().oracle_compute_effective_scale(bs, ws2, ins)


def e4m3_to_f32(b: int) -> float:
    return lib().oracle_e4m3_to_f32(b)


def e4m3_table() -> np.ndarray:
    return np.array([e4m3_to_f32(b) for b in range(256)], dtype=np.float32)


def f32_to_e4m3(x: float) -> int:
    return lib().oracle_f32_to_e4m3_satfinite(x)


def f32_to_e2m1(x: float) -> int:
    return lib().oracle_f32_to_e2m1_satfinite(x)


def sigmoid(x: float) -> float:
    return lib().oracle_sigmoid(x)


def silu(x: float) -> float:
    return lib().oracle_silu(x)


def dequant_tile(packed, scales, weight_stride, scale_stride, start_row, start_col,
                 tile_m, tile_k):
    """nvfp4/nvfp4_gemm_gpu.mojo:44-96."""
    packed, scales = _u8(packed), _u8(scales)
    out = np.empty((tile_m, tile_k), dtype=np.float32)
    lib().oracle_dequant_tile(_p(packed, _u8p), _p(scales, _u8p), _p(out, _f32p),
                              weight_stride, scale_stride, start_row, start_col,
                              tile_m, tile_k)
    return out


def dequant(packed, scales):
    """Full-matrix dequant: LUT * float(sf), fp32 [N, K]."""
    packed = _u8(packed)
    N, Kh = packed.shape
    return dequant_tile(packed, scales, Kh, Kh * 2 // 16, 0, 0, N, Kh * 2)


def matvec(packed, scales, x, input_scale=1.0, ws2=1.0, ws2_rows=None):
    """nvfp4/deltanet.mojo:549-584 for one fp32 vector x [K] -> y [N]."""
    packed, scales, x = _u8(packed), _u8(scales), _f32(x)
    N, Kh = packed.shape
    y = np.empty(N, dtype=np.float32)
    wr = None if ws2_rows is None else _f32(ws2_rows)
    lib().oracle_matvec(Kh * 2, N, input_scale, ws2, _p(wr, _f32p), _p(packed, _u8p),
                        _p(scales, _u8p), _p(x, _f32p), _p(y, _f32p))
    return y


def linear(packed, scales, x, input_scale=1.0, ws2=1.0, ws2_rows=None,
           rows=None, cols=None, n_threads=1):
    """Token-major linear y[M, N] (or the rows x cols sample), fp32."""
    packed, scales, x = _u8(packed), _u8(scales), _f32(x)
    N, Kh = packed.shape
    M = x.shape[0]
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    c = None if cols is None else np.ascontiguousarray(cols, dtype=np.int64)
    R = M if r is None else len(r)
    C = N if c is None else len(c)
    y = np.empty((R, C), dtype=np.float32)
    wr = None if ws2_rows is None else _f32(ws2_rows)
    lib().oracle_linear(M, Kh * 2, N, input_scale, ws2, _p(wr, _f32p),
                        _p(packed, _u8p), _p(scales, _u8p), _p(x, _f32p), _p(y, _f32p),
                        _p(r, _i64p), 0 if r is None else len(r),
                        _p(c, _i64p), 0 if c is None else len(c), int(n_threads))
    return y


def gemm_kernel(packed, scales, act_kmajor, alpha):
    """nvfp4/nvfp4_gemm_gpu.mojo:99-182: out[M_out, N_tok] from act[K, N_tok]."""
    packed, scales, act = _u8(packed), _u8(scales), _f32(act_kmajor)
    M_out, Kh = packed.shape
    K, N_tok = act.shape
    out = np.empty((M_out, N_tok), dtype=np.float32)
    lib().oracle_gemm_kernel(M_out, N_tok, K, _p(packed, _u8p), _p(scales, _u8p),
                             _p(act, _f32p), _p(out, _f32p), alpha)
    return out


def quantize_act(x, input_scale):
    x = _f32(x)
    M, K = x.shape
    q = np.empty((M, K // 2), dtype=np.uint8)
    s = np.empty((M, K // 16), dtype=np.uint8)
    lib().oracle_quantize_act(M, K, _p(x, _f32p), input_scale, _p(q, _u8p), _p(s, _u8p))
    return q, s


def linear_w4a4(packed, scales, x, input_scale, ws2=1.0, ws2_rows=None, rows=None, cols=None,
                n_threads=1):
    """W4A4 linear: x quantized to NVFP4 with input_scale (quantize_act), then
    y = input_scale * ws2 * dequant(W) @ dequant(Xq)^T in fp32 (linear on
    the dequantized activations)."""
    q, s = quantize_act(_f32(x), input_scale)
    return linear(packed, scales, dequant(q, s), input_scale=input_scale, ws2=ws2,
                  ws2_rows=ws2_rows, rows=rows, cols=cols, n_threads=n_threads)


def fp4_digits(x, digits=4):
    """FP4-digit decomposition of activations (the decode GEMV draft's
    input side; no reference counterpart): per token t and digit d,
    s[t, d] = amax(residual_t) / (6 * 448), digit = quantize_act(residual_t,
    s[t, d]) (per-16 E4M3 scales, E2M1 codes, RNE), residual_t -=
    dequant(digit) * s[t, d].  Returns codes [M * D, K/2], scales
    [M * D, K/16] and s [M * D] with row t * D + d."""
    x = _f32(x)
    M, K = x.shape
    codes = np.zeros((M * digits, K // 2), np.uint8)
    scs = np.zeros((M * digits, K // 16), np.uint8)
    sd = np.zeros(M * digits, np.float32)
    for t in range(M):
        r = x[t:t + 1].copy()
        for d in range(digits):
            s_ = np.float32(np.abs(r).max()) / np.float32(6.0 * 448.0)
            row = t * digits + d
            sd[row] = s_
            if s_ == 0.0:
                continue
            q, sc = quantize_act(r, float(s_))
            codes[row], scs[row] = q[0], sc[0]
            r = (r - dequant(q, sc) * s_).astype(np.float32)
    return codes, scs, sd


def fp4_digits_value(codes, scales, sd, digits=4):
    """The activations the digits represent: [M, K] fp32."""
    v = dequant(codes, scales) * sd[:, None]
    return v.reshape(-1, digits, v.shape[1]).sum(axis=1, dtype=np.float32)


def router(x, router_w):
    x, r = _f32(x), _f32(router_w)
    T, H = x.shape
    E = r.shape[1]
    logits = np.empty((T, E), dtype=np.float32)
    probs = np.empty((T, E), dtype=np.float32)
    lib().oracle_router(T, H, E, _p(x, _f32p), _p(r, _f32p), _p(logits, _f32p),
                        _p(probs, _f32p))
    return logits, probs


def moe(x, w, top_k=8, renormalize=True, tokens=None, force_ids=None, n_threads=1):
    """One MoE FFN layer; `w` is a dict of stacked expert tensors (numpy).

    Keys: router [H, E] f32, gu_w [E, 2I, H/2] u8, gu_sf [E, 2I, H/16] u8,
    gu_ws2 [E, 2I] f32, gu_in [E] f32 (optional), dn_w [E, H, I/2] u8,
    dn_sf [E, H, I/16] u8, dn_ws2 [E, H] f32, dn_in [E] f32 (optional).
    Returns (out [R, H] f32, topk_ids [R, k] i32, topk_w [R, k] f32).
    """
    x = _f32(x)
    T, H = x.shape
    E = w["router"].shape[1]
    I = w["gu_w"].shape[1] // 2
    tok = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int64)
    R = T if tok is None else len(tok)
    out = np.empty((R, H), dtype=np.float32)
    ids = np.empty((R, top_k), dtype=np.int32)
    tw = np.empty((R, top_k), dtype=np.float32)
    fi = None if force_ids is None else np.ascontiguousarray(force_ids, dtype=np.int32)
    g = {k: (_f32(v) if v is not None and v.dtype != np.uint8 else v) for k, v in w.items()}
    lib().oracle_moe(T, H, I, E, top_k, int(renormalize), _p(x, _f32p),
                     _p(g["router"], _f32p), _p(_u8(g["gu_w"]), _u8p),
                     _p(_u8(g["gu_sf"]), _u8p), _p(g["gu_ws2"], _f32p),
                     _p(g.get("gu_in"), _f32p), _p(_u8(g["dn_w"]), _u8p),
                     _p(_u8(g["dn_sf"]), _u8p), _p(g["dn_ws2"], _f32p),
                     _p(g.get("dn_in"), _f32p), _p(out, _f32p),
                     _p(tok, _i64p), 0 if tok is None else len(tok),
                     _p(ids, _i32p), _p(tw, _f32p), _p(fi, _i32p), int(n_threads))
    return out, ids, tw


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# Gated DeltaNet decode step (nvfp4/deltanet.mojo:51-542)
# ---------------------------------------------------------------------------

def softplus(x: float) -> float:
    """nvfp4/deltanet.mojo:56-63."""
    return lib().oracle_softplus(x)


def dn_matvec(mat, vec):
    """matvec (nvfp4/deltanet.mojo:239-254): mat [rows, cols] @ vec [cols]."""
    mat, vec = _f32(mat), _f32(vec)
    out = np.empty(mat.shape[0], dtype=np.float32)
    lib().oracle_dn_matvec(_p(mat, _f32p), _p(vec, _f32p), _p(out, _f32p), *mat.shape)
    return out


def dn_matvec_t(mat, vec):
    """matvec_transposed (nvfp4/deltanet.mojo:221-236): mat^T @ vec."""
    mat, vec = _f32(mat), _f32(vec)
    out = np.empty(mat.shape[1], dtype=np.float32)
    lib().oracle_dn_matvec_t(_p(mat, _f32p), _p(vec, _f32p), _p(out, _f32p), *mat.shape)
    return out


def rms_norm(x, eps=1e-6):
    """rms_norm_inplace (nvfp4/deltanet.mojo:270-284), on a copy."""
    y = _f32(x).copy()
    lib().oracle_rms_norm(_p(y, _f32p), y.size, eps)
    return y


def conv1d_step(new_input, buf, w, bias=None):
    """conv1d_step (nvfp4/deltanet.mojo:287-328); buf [ch, k-1] updated in place."""
    x, w = _f32(new_input), _f32(w)
    assert buf.dtype == np.float32 and buf.flags.c_contiguous
    ch, kernel = w.shape
    out = np.empty(ch, dtype=np.float32)
    b = None if bias is None else _f32(bias)
    lib().oracle_conv1d_step(_p(x, _f32p), _p(buf, _f32p), _p(w, _f32p), _p(out, _f32p), ch,
                             kernel, _p(b, _f32p))
    return out


def deltanet_state(cfg):
    """Zero DeltaNetState (nvfp4/deltanet.mojo:181-218): s [nvh, kd, vd] and the
    conv windows [dim, conv_k - 1] of q, k, v."""
    nkh, nvh, kd, vd, ck = (cfg["num_key_heads"], cfg["num_value_heads"], cfg["key_dim"],
                            cfg["value_dim"], cfg["conv_kernel"])
    z = lambda *s: np.zeros(s, dtype=np.float32)
    return {"s": z(nvh, kd, vd), "q": z(nkh * kd, ck - 1), "k": z(nkh * kd, ck - 1),
            "v": z(nvh * vd, ck - 1)}


def deltanet_forward(cfg, hidden, w, state):
    """deltanet_forward (nvfp4/deltanet.mojo:335-546) for one token with fp32
    weights (for NVFP4 projections, pass their dequantized matrices times
    alpha: the dequantization is exact in fp32).  `w` keys: qkv, z, b, a,
    out, a_log, dt_bias, conv_q, conv_k, conv_v and optional conv_bias_q/k/v;
    `state` (deltanet_state) is updated in place.  Returns out [d_model]."""
    d = cfg["d_model"]
    out = np.empty(d, dtype=np.float32)
    g = {k: (None if v is None else _f32(v)) for k, v in w.items()}
    for k_ in ("s", "q", "k", "v"):
        assert state[k_].dtype == np.float32 and state[k_].flags.c_contiguous
    lib().oracle_deltanet_forward(
        d, cfg["num_key_heads"], cfg["num_value_heads"], cfg["key_dim"], cfg["value_dim"],
        cfg["conv_kernel"], cfg.get("rms_eps", 1e-6), _p(_f32(hidden), _f32p), _p(out, _f32p),
        _p(g["qkv"], _f32p), _p(g["z"], _f32p), _p(g["b"], _f32p), _p(g["a"], _f32p),
        _p(g["out"], _f32p), _p(g["a_log"], _f32p), _p(g["dt_bias"], _f32p),
        _p(g["conv_q"], _f32p), _p(g["conv_k"], _f32p), _p(g["conv_v"], _f32p),
        _p(g.get("conv_bias_q"), _f32p), _p(g.get("conv_bias_k"), _f32p),
        _p(g.get("conv_bias_v"), _f32p), _p(state["s"], _f32p), _p(state["q"], _f32p),
        _p(state["k"], _f32p), _p(state["v"], _f32p))
    return out
