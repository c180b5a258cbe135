"""The DeltaNet oracle (oracle/nvfp4_oracle.c, restating nvfp4/deltanet.mojo)
pinned against every known answer of the reference's tests/test_deltanet.mojo,
with that file's tolerance rule (tests/helpers.mojo:7-19: absolute or
relative difference within tol).  CPU only."""
import numpy as np
import pytest


def approx_eq(a, b, tol=1e-4):
    """approx_eq (tests/helpers.mojo:7-19)."""
    diff = abs(float(a) - float(b))
    if diff <= tol:
        return True
    denom = abs(max(float(a), float(b)))
    return denom > 0.0 and diff / denom <= tol


def expect_close(actual, expected, tol=1e-4):
    assert approx_eq(np.float32(actual), np.float32(expected), tol), (actual, expected)


def test_activations(O):
    """tests/test_deltanet.mojo:57-80."""
    expect_close(O.softplus(0.0), 0.6931472)
    expect_close(O.softplus(30.0), 30.0)
    expect_close(O.softplus(-30.0), 0.0)
    expect_close(O.softplus(1.0), 1.3132616)
    expect_close(O.sigmoid(0.0), 0.5)
    expect_close(O.sigmoid(10.0), 0.9999546)
    expect_close(O.sigmoid(-10.0), 4.539787e-05)
    expect_close(O.silu(0.0), 0.0)
    expect_close(O.silu(1.0), 0.7310586)
    expect_close(O.silu(-1.0), -0.26894143)


def test_linear_algebra(O):
    """tests/test_deltanet.mojo:84-159."""
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    y = O.dn_matvec(a, np.ones(3, np.float32))
    expect_close(y[0], 6.0)
    expect_close(y[1], 15.0)
    yt = O.dn_matvec_t(a.reshape(3, 2), np.ones(3, np.float32))
    expect_close(yt[0], 9.0)
    expect_close(yt[1], 12.0)
    x = O.rms_norm(np.array([1, 2, 3, 4], np.float32), 1e-6)
    r = np.sqrt(np.float32(7.5))
    for i in range(4):
        expect_close(x[i], (i + 1) / r)


def test_conv1d_step(O):
    """tests/test_deltanet.mojo:163-215."""
    buf = np.array([[0.5, 1.0], [0.2, 0.3]], np.float32)
    w = np.array([[1.0, 2.0, 3.0], [0.5, 1.5, 2.5]], np.float32)
    out = O.conv1d_step(np.array([2.0, 4.0], np.float32), buf, w)
    expect_close(out[0], 8.5)
    expect_close(out[1], 10.55)
    expect_close(buf[0, 0], 1.0)
    expect_close(buf[0, 1], 2.0)
    expect_close(buf[1, 0], 0.3)
    expect_close(buf[1, 1], 4.0)


def identity_like(rows, cols, scale):
    """make_identity_like (tests/test_deltanet.mojo:41-50)."""
    m = np.zeros((rows, cols), np.float32)
    m[np.arange(rows), np.arange(rows) % cols] = scale
    return m


def small_case():
    """The small configuration and weights of test_forward_small
    (tests/test_deltanet.mojo:285-346)."""
    cfg = dict(d_model=8, num_key_heads=2, num_value_heads=2, key_dim=4, value_dim=4,
               conv_kernel=4, rms_eps=1e-6)
    d, nvh, qd, kd, vd, ck = 8, 2, 8, 8, 8, 4
    conv = lambda ch: np.concatenate([np.zeros((ch, ck - 1), np.float32),
                                      np.ones((ch, 1), np.float32)], 1)
    w = dict(qkv=identity_like(24, d, 0.1), z=identity_like(8, d, 0.5),
             b=np.full((nvh, d), 0.1, np.float32), a=np.full((nvh, d), 0.05, np.float32),
             out=identity_like(d, 8, 1.0), a_log=np.array([0.0, 0.5], np.float32),
             dt_bias=np.array([0.0, 0.1], np.float32), conv_q=conv(qd), conv_k=conv(kd),
             conv_v=conv(vd))
    hidden = (np.float32(0.1) + np.arange(d, dtype=np.float32) * np.float32(0.1))
    return cfg, w, hidden


def test_forward_small_golden(O):
    """test_forward_small (tests/test_deltanet.mojo:285-425): result[0] and
    result[7] of the first step, state updated, the second step differs."""
    cfg, w, hidden = small_case()
    st = O.deltanet_state(cfg)
    r1 = O.deltanet_forward(cfg, hidden, w, st)
    assert np.any(r1 != 0.0)
    expect_close(r1[0], 5.879743e-05, 1e-6)
    expect_close(r1[7], 0.0271918, 1e-5)
    assert np.any(st["s"] != 0.0)
    r2 = O.deltanet_forward(cfg, hidden, w, st)
    assert np.any(r1 != r2)


def test_config_sizes():
    """test_config / test_state_init / test_o1_memory
    (tests/test_deltanet.mojo:219-445): the default layer's dimensions,
    through the Python mirror's DeltaNetConfig and DeltaNetState."""
    from nvfp4.deltanet import DeltaNetConfig, DeltaNetState

    c = DeltaNetConfig()
    assert (c.d_model, c.num_key_heads, c.num_value_heads, c.key_dim, c.value_dim,
            c.conv_kernel) == (2048, 16, 32, 128, 128, 4)
    assert c.total_qkv_dim() == 8192
    assert c.z_dim() == 4096 and c.v_dim() == 4096
    assert c.q_dim() == c.k_dim() == 2048
    assert c.v_groups() == 2
    assert c.state_size_per_head() == 16384
    assert c.total_state_floats() == 524288
    assert c.total_state_floats() * 4 == 2097152  # state bytes per layer
    st = DeltaNetState(c, batch=2, device="cpu")
    assert tuple(st.s_matrix.shape) == (2, 32, 128, 128) and not st.s_matrix.any()
    assert tuple(st.conv_buf_q.shape) == (2, 2048, 3)
    assert tuple(st.conv_buf_v.shape) == (2, 4096, 3)


def test_host_softplus_matches_oracle(O):
    """nvfp4.deltanet.softplus (host-side mirror) against the oracle's."""
    from nvfp4.deltanet import softplus

    for x in (-30.0, -20.5, -1.0, 0.0, 0.5, 1.0, 19.9, 20.5, 30.0):
        expect_close(softplus(x), O.softplus(x), 1e-6)


def dn_shape_ok(d_model, nkh, nvh, kd, vd, ck, eps):
    """The shapes nvfp4_deltanet_forward serves (include/nvfp4_deltanet.h)."""
    return (d_model > 0 and d_model % 16 == 0 and nkh > 0 and nvh > 0 and nvh % nkh == 0
            and 0 < kd <= 256 and 4 <= vd <= 256 and vd & (vd - 1) == 0 and 1 <= ck <= 8
            and (nvh * vd) % 16 == 0 and eps >= 0.0)


def test_descriptor_rules_without_gpu():
    """nvfp4_deltanet_workspace_size is 0 exactly for the shapes the header
    rules out (host-side check, no GPU), over generated descriptors, for
    B >= 1 sequences (B = 0 needs no workspace at all)."""
    import ctypes

    from hypothesis import given, settings
    from hypothesis import strategies as st
    from nvfp4 import _lib

    L = _lib.load()

    @settings(max_examples=400, deadline=None)
    @given(st.integers(-16, 4096), st.integers(-1, 9), st.integers(-1, 40), st.integers(-1, 300),
           st.sampled_from([-4, 0, 2, 3, 4, 8, 12, 16, 32, 64, 96, 128, 256, 512]),
           st.integers(-1, 10), st.sampled_from([1e-6, 0.0, -1e-6]), st.integers(1, 3))
    def check(d_model, nkh, nvh, kd, vd, ck, eps, B):
        desc = _lib.DeltaNetDesc(d_model, nkh, nvh, kd, vd, ck, eps)
        size = L.nvfp4_deltanet_workspace_size(ctypes.byref(desc), B)
        assert (size > 0) == dn_shape_ok(d_model, nkh, nvh, kd, vd, ck, eps), desc

    check()


def test_forward_argument_checks_without_gpu():
    """nvfp4_deltanet_forward refuses bad arguments before any CUDA work."""
    import ctypes

    from nvfp4 import _lib

    L = _lib.load()
    desc = _lib.DeltaNetDesc(2048, 16, 32, 128, 128, 4, 1e-6)
    w = _lib.DeltaNetWeightPtrs()
    st = _lib.DeltaNetStatePtrs()

    def call(B=1, hdt=1, odt=1, pdt=1, ws=256, ws_bytes=1 << 40, weights=w, state=st):
        return L.nvfp4_deltanet_forward(ctypes.byref(desc), ctypes.byref(weights), 256, hdt, 256,
                                        odt, B, ctypes.byref(state), pdt, ws, ws_bytes, None)

    assert call() == _lib.NVFP4_ERR_INVALID_ARG  # null weight pointers
    for name in ("a_log", "dt_bias", "conv_q", "conv_k", "conv_v"):
        setattr(w, name, 256)
    for name in ("s", "conv_q", "conv_k", "conv_v"):
        setattr(st, name, 256)
    w.conv_bias_q = 256  # one bias of three
    assert call() == _lib.NVFP4_ERR_INVALID_ARG
    assert b"biases" in L.nvfp4_last_error_string()
    w.conv_bias_q = None
    assert call(hdt=7) == _lib.NVFP4_ERR_INVALID_ARG
    assert call(ws=16) == _lib.NVFP4_ERR_INVALID_ARG  # workspace not 256-byte aligned
    assert call(B=-1) == _lib.NVFP4_ERR_INVALID_ARG
    assert call(B=0) == _lib.NVFP4_OK  # nothing to do
    assert call(ws_bytes=1024) == _lib.NVFP4_ERR_WORKSPACE
