"""GPU parity of the NVFP4 dequant / GEMV / linear kernels against the CPU
oracle, through the C ABI (via the nvfp4 Python mirror).

Tolerances: dequant bit-exact (incl. -0.0 and NaN); GEMV/GEMM
max|err| <= 2e-2 * RMS(ref) for bf16 operands with fp32 accumulation; the
fp32-activation path (nvfp4_matvec arithmetic) <= 1e-5 * RMS(ref).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2
TOL_F32 = 1e-5


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.abs(got - ref).max() / rms)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def exhaustive_weights():
    """256 rows (row r uses blockscale code r in every group) x K = 256 with
    each 16-group holding codes 0..15 in k order (low nibble = even k)."""
    rows, K = 256, 256
    codes = np.tile(np.arange(16, dtype=np.uint8), (rows, K // 16))
    w = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    sf = np.repeat(np.arange(256, dtype=np.uint8)[:, None], K // 16, axis=1)
    return w, sf


def bits32(a):
    a = np.asarray(a, np.float32).copy()
    nan = np.isnan(a)
    b = a.view(np.uint32).copy()
    b[nan] = 0x7FC00000
    return b


def test_dequant_fp32_bit_exact_all_codes(O, cuda):
    import nvfp4

    w, sf = exhaustive_weights()
    ref = O.dequant(w, sf)
    got = nvfp4.dequant(dev(w), dev(sf), torch.float32).cpu().numpy()
    assert np.array_equal(bits32(got), bits32(ref))
    assert np.signbit(got[0, 8]) and got[0, 8] == 0.0  # code 8 -> -0.0
    # Into a caller buffer (the form the dequant microbenchmark uses).
    out = torch.full(ref.shape, float("nan"), dtype=torch.float32, device=cuda)
    nvfp4.dequant(dev(w), dev(sf), out=out)
    assert np.array_equal(bits32(out.cpu().numpy()), bits32(ref))


def test_dequant_bf16_bit_exact_all_codes(O, cuda):
    """The bf16 form is the tensor-core operand decode (LUT*scale*2^-7, then
    *2^7): it must equal the exact fp32 dequant rounded to bf16 (which is
    exact), sign of zero and NaN included."""
    import nvfp4

    w, sf = exhaustive_weights()
    ref = torch.from_numpy(O.dequant(w, sf)).to(torch.bfloat16).view(torch.int16).numpy()
    got = nvfp4.dequant(dev(w), dev(sf), torch.bfloat16).cpu()
    gb = got.view(torch.int16).numpy().copy()
    isnan = torch.isnan(got.float()).numpy()
    assert np.array_equal(isnan, np.isnan(O.dequant(w, sf)))
    assert np.array_equal(gb[~isnan], ref[~isnan])


def test_dequant_tile_matches_reference_form(O, cuda):
    import nvfp4
    from nvfp4 import synthetic

    N, K = 1536, 2048
    wd = synthetic.linear_weights(N, K, seed=0)
    out = torch.empty((7, 64), dtype=torch.float32, device=cuda)
    nvfp4.load_and_dequant_fp4_tile(dev(wd["w"]), dev(wd["sf"]), out, K // 2, K // 16,
                                    5, 48, 7, 64)
    ref = O.dequant_tile(wd["w"], wd["sf"], K // 2, K // 16, 5, 48, 7, 64)
    assert np.array_equal(bits32(out.cpu().numpy()), bits32(ref))


def test_config0_fp32_linear_and_matvec(O, cuda):
    """Single NVFP4 linear, fp32 x [4, 2048], W [1536, 1024]: the fp32 path
    (nvfp4_matvec arithmetic), scalar and per-row weight_scale_2."""
    import nvfp4
    from nvfp4 import synthetic

    N, K, M = 1536, 2048, 4
    wd = synthetic.linear_weights(N, K, seed=0)
    x = synthetic.activations(M, K, seed=1)
    W, SF, X = dev(wd["w"]), dev(wd["sf"]), dev(x)
    lin = nvfp4.NvFp4Linear(K, N, input_scale=1.0, weight_scale_2=1.0,
                            weight_scale_2_rows=dev(wd["ws2"]))
    y = torch.empty((M, N), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, W, SF, X, y, M)
    ref = O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"])
    assert rel_err(y.cpu().numpy(), ref) <= TOL_F32
    lin_s = nvfp4.NvFp4Linear(K, N, input_scale=0.5, weight_scale_2=0.003)
    r = torch.empty(N, dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_matvec(lin_s, W, SF, X[2].contiguous(), r)
    ref2 = O.matvec(wd["w"], wd["sf"], x[2], input_scale=0.5, ws2=0.003)
    assert rel_err(r.cpu().numpy(), ref2) <= TOL_F32


@pytest.mark.parametrize("K,N", [(2048, 1536), (768, 2048), (4096, 14336)])
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_decode_gemv_sweep(O, cuda, K, N, M):
    """Decode GEMV sweep: bf16 x, the M <= 8 decode path, fp32 and bf16 out."""
    import nvfp4
    from nvfp4 import synthetic

    wd = synthetic.linear_weights(N, K, seed=100 + K + N)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=M))
    lin = nvfp4.NvFp4Linear(K, N, weight_scale_2_rows=dev(wd["ws2"]))
    W, SF, X = dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16)
    y32 = torch.empty((M, N), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, W, SF, X, y32, M, flags=nvfp4._lib.FLAG_FORCE_SKINNY)
    ybf = nvfp4.nvfp4_linear(lin, W, SF, X)
    ref = O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"])
    # Exact decode + fp32 accumulation: only summation order differs.
    assert rel_err(y32.cpu().numpy(), ref) <= 1e-5
    assert rel_err(ybf.float().cpu().numpy(), ref) <= TOL_BF16
    # The tcgen05 GEMV (opt-in) agrees with the oracle too.
    yt = torch.empty((M, N), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, W, SF, X, yt, M, flags=nvfp4._lib.FLAG_TS_GEMV)
    assert rel_err(yt.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("N,K,M", [(100, 512, 1), (100, 512, 3), (136, 768, 8), (64, 256, 5),
                                   (1000, 4096, 7), (24, 2048, 2)])
def test_decode_gemv_shapes(O, cuda, N, K, M):
    """Decode GEMV (M <= 8, K % 256 == 0): ragged N, K slices of 1 to 8 chunks
    per cluster rank; fp32 and bf16 outputs, scalar alpha."""
    import nvfp4
    from nvfp4 import synthetic

    wd = synthetic.linear_weights(N, K, seed=N + K + M)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=M + 3))
    lin = nvfp4.NvFp4Linear(K, N, input_scale=0.75, weight_scale_2=0.004)
    W, SF, X = dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16)
    y32 = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, W, SF, X, y32, M)
    ybf = nvfp4.nvfp4_linear(lin, W, SF, X)
    ref = O.linear(wd["w"], wd["sf"], x, input_scale=0.75, ws2=0.004)
    assert not torch.isnan(y32).any()
    assert rel_err(y32.cpu().numpy(), ref) <= 1e-5
    assert rel_err(ybf.float().cpu().numpy(), ref) <= TOL_BF16
    # The tcgen05 GEMV (opt-in) on the same ragged shapes.
    yt = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, W, SF, X, yt, M, flags=nvfp4._lib.FLAG_TS_GEMV)
    assert not torch.isnan(yt).any()
    assert rel_err(yt.cpu().numpy(), ref) <= 1e-5


def test_decode_gemv_chained_layers(O, cuda):
    """Two decode GEMVs in a chain (the second reads the first's output),
    three times in a row on one stream with new inputs and reused buffers:
    the kernel starts before its predecessor has finished (programmatic
    dependent launch), so it must never see a previous iteration's data."""
    import nvfp4
    from nvfp4 import synthetic

    M, K, N = 4, 2048, 1536
    wa = synthetic.linear_weights(N, K, seed=61)
    wb = synthetic.linear_weights(K, N, seed=62)
    la = nvfp4.NvFp4Linear(K, N, weight_scale_2_rows=dev(wa["ws2"]))
    lb = nvfp4.NvFp4Linear(N, K, weight_scale_2_rows=dev(wb["ws2"]))
    Wa, Sa, Wb, Sb = dev(wa["w"]), dev(wa["sf"]), dev(wb["w"]), dev(wb["sf"])
    X = torch.empty((M, K), dtype=torch.bfloat16, device=cuda)
    Y1 = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    Y2 = torch.empty((M, K), dtype=torch.float32, device=cuda)
    xs = [synthetic.bf16_round(synthetic.activations(M, K, seed=70 + i)) * (1 + 3 * i)
          for i in range(3)]
    y1s, y2s = [], []
    for x in xs:
        X.copy_(torch.from_numpy(x).to(torch.bfloat16))
        nvfp4.nvfp4_linear_forward(la, Wa, Sa, X, Y1, M)
        nvfp4.nvfp4_linear_forward(lb, Wb, Sb, Y1, Y2, M)
        y1s.append(Y1.clone())
        y2s.append(Y2.clone())
    torch.cuda.synchronize()
    for i, x in enumerate(xs):
        y1 = y1s[i].float().cpu().numpy()
        assert rel_err(y1, O.linear(wa["w"], wa["sf"], x, ws2_rows=wa["ws2"])) <= TOL_BF16, i
        ref2 = O.linear(wb["w"], wb["sf"], y1, ws2_rows=wb["ws2"])
        assert rel_err(y2s[i].cpu().numpy(), ref2) <= 1e-5, i


def test_decode_gemv_activation_range(O, cuda):
    """Per-token power-of-two scaling of the f16 activations: tokens far
    outside the f16 range (|x| ~ 1e30, 1e-30), an all-zero token, and
    ordinary ones in one call, each exact to fp32 summation order."""
    import nvfp4
    from nvfp4 import synthetic

    N, K = 96, 1024
    scales = [1.0, 1e30, 1e-30, 0.0, 3e4, 1e-6]
    M = len(scales)
    wd = synthetic.linear_weights(N, K, seed=77)
    x = synthetic.activations(M, K, seed=78) * np.asarray(scales, np.float32)[:, None]
    x = synthetic.bf16_round(x)
    lin = nvfp4.NvFp4Linear(K, N)
    y = torch.empty((M, N), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16), y, M)
    y = y.cpu().numpy()
    ref = O.linear(wd["w"], wd["sf"], x)
    for t, sc in enumerate(scales):
        if sc == 0.0:
            assert (y[t] == 0).all()
        else:
            assert rel_err(y[t], ref[t]) <= 1e-5, (t, sc)


@pytest.mark.parametrize("M", [3, 13, 17, 33, 64])
def test_skinny_ragged_shapes(O, cuda, M):
    """N not a multiple of 16, K % 128 == 64 (a partial last round), several
    token items."""
    import nvfp4
    from nvfp4 import synthetic

    N, K = 100, 64 * 5
    wd = synthetic.linear_weights(N, K, seed=M)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=M + 1))
    lin = nvfp4.NvFp4Linear(K, N, input_scale=1.5, weight_scale_2=0.01)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16), y, M)
    ref = O.linear(wd["w"], wd["sf"], x, input_scale=1.5, ws2=0.01)
    assert not torch.isnan(y).any()  # every output written
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5


def test_fp32_path_odd_k(O, cuda):
    """K % 64 != 0 goes to the CUDA-core fp32 path (any K multiple of 16)."""
    import nvfp4
    from nvfp4 import synthetic

    N, K, M = 40, 48, 5
    wd = synthetic.linear_weights(N, K, seed=9)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=10))
    lin = nvfp4.NvFp4Linear(K, N)
    y = nvfp4.nvfp4_linear(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16),
                           out_dtype=torch.float32)
    ref = O.linear(wd["w"], wd["sf"], x)
    assert rel_err(y.cpu().numpy(), ref) <= TOL_F32


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_gemm_kernel_reference_layout(O, cuda, dt):
    """nvfp4_gemm_kernel: act [K, N_tok] -> out [M_out, N_tok] (reference layout)."""
    import nvfp4
    from nvfp4 import synthetic

    M_out, K, N_tok = 256, 512, 6
    wd = synthetic.linear_weights(M_out, K, seed=21)
    x = synthetic.bf16_round(synthetic.activations(N_tok, K, seed=22))
    act = dev(np.ascontiguousarray(x.T), dt)
    out = torch.empty((M_out, N_tok), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_gemm_kernel(dev(wd["w"]), dev(wd["sf"]), act, out, alpha=0.125)
    ref = O.gemm_kernel(wd["w"], wd["sf"], np.ascontiguousarray(x.T), 0.125)
    assert rel_err(out.cpu().numpy(), ref) <= TOL_F32


def test_nan_scale_propagates_and_empty_batch(O, cuda):
    import nvfp4
    from nvfp4 import synthetic

    N, K, M = 32, 128, 2
    wd = synthetic.linear_weights(N, K, seed=5)
    wd["sf"][3, 2] = 0x7F  # NaN blockscale in row 3
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=6))
    lin = nvfp4.NvFp4Linear(K, N)
    y = nvfp4.nvfp4_linear(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16),
                           out_dtype=torch.float32).cpu().numpy()
    assert np.isnan(y[:, 3]).all()
    assert not np.isnan(np.delete(y, 3, axis=1)).any()
    empty = torch.empty((0, N), dtype=torch.bfloat16, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, dev(wd["w"]), dev(wd["sf"]),
                               torch.empty((0, K), dtype=torch.bfloat16, device=cuda), empty, 0)
    torch.cuda.synchronize()


@pytest.mark.parametrize("N,K,M", [(256, 512, 65), (256, 512, 256), (200, 256, 300),
                                   (384, 1024, 513), (128, 768, 97), (1024, 256, 2560)])
def test_tc_gemm_small_shapes(O, cuda, N, K, M):
    """tcgen05 W4A16 GEMM (forced): ragged N, M not a multiple of the tile,
    a single blockscale chunk (K = 256), an odd number of chunks (K = 768),
    and more tiles than SMs (persistent CTAs, both accumulator buffers); fp32
    out checked against the oracle."""
    import nvfp4
    from nvfp4 import synthetic

    wd = synthetic.linear_weights(N, K, seed=N + K + M)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=M))
    lin = nvfp4.NvFp4Linear(K, N, input_scale=0.5, weight_scale_2_rows=dev(wd["ws2"]))
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16), y, M,
                               flags=nvfp4._lib.FLAG_FORCE_TC)
    torch.cuda.synchronize()
    assert nvfp4._lib.load().nvfp4_device_status() == 0
    ref = O.linear(wd["w"], wd["sf"], x, input_scale=0.5, ws2_rows=wd["ws2"])
    got = y.cpu().numpy()
    assert not np.isnan(got).any()
    assert rel_err(got, ref) <= 1e-5


@pytest.mark.parametrize("M", [512, 2048, 8192])
def test_prefill_w4a16_config2_sampled(O, cuda, M):
    """Prefill W4A16 at the benchmark shape (K=4096, N=14336): bf16 out,
    oracle on a sample of tokens x output features."""
    import nvfp4
    from nvfp4 import synthetic

    N, K = 14336, 4096
    wd = synthetic.linear_weights(N, K, seed=2)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=3))
    lin = nvfp4.NvFp4Linear(K, N, weight_scale_2_rows=dev(wd["ws2"]))
    y = nvfp4.nvfp4_linear(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16))
    torch.cuda.synchronize()
    assert nvfp4._lib.load().nvfp4_device_status() == 0
    rng = np.random.default_rng(M)
    rows = np.sort(rng.choice(M, 24, replace=False))
    cols = np.sort(rng.choice(N, 256, replace=False))
    ref = O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"], rows=rows, cols=cols, n_threads=8)
    got = y.float().cpu().numpy()[np.ix_(rows, cols)]
    assert rel_err(got, ref) <= TOL_BF16
    # fp32 output agrees with the oracle to fp32 summation-order error (the
    # oracle sums K = 4096 terms sequentially; 200x tighter than the bf16 bar).
    y32 = torch.empty((M, N), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16), y32, M)
    assert rel_err(y32.cpu().numpy()[np.ix_(rows, cols)], ref) <= 1e-4


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_decode_gemv_repeatable(cuda, M):
    """Repeated calls are bitwise identical (fixed reduction order, and every
    staged weight chunk is read before TMA refills its buffer): 20 calls of
    the K=4096, N=14336 decode GEMV, fp32 out."""
    import nvfp4
    from nvfp4 import synthetic

    K, N = 4096, 14336
    wd = synthetic.linear_weights_cuda(N, K, seed=5 + M)
    x = torch.randn((M, K), device=cuda).to(torch.bfloat16)
    lin = nvfp4.NvFp4Linear(K, N, weight_scale_2_rows=wd["ws2"])
    outs = []
    for _ in range(20):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
        nvfp4.nvfp4_linear_forward(lin, wd["w"], wd["sf"], x, y, M)
        outs.append(y)
    first = outs[0]
    assert not torch.isnan(first).any()
    for i, y in enumerate(outs[1:], 1):
        assert torch.equal(y, first), f"call {i} differs"


DIGIT_TOL = 1e-3  # four FP4 digits: ~5e-4 of RMS measured against the exact linear


@pytest.mark.parametrize("K,N", [(2048, 1536), (768, 2048), (4096, 14336), (512, 100),
                                 (1024, 136), (4096, 1000)])
@pytest.mark.parametrize("M", [1, 3, 8])
def test_digit_gemv_against_oracle(O, cuda, K, N, M):
    """NVFP4_FLAG_DIGIT_GEMV: activations as four NVFP4 digits, weights as
    stored into block-scaled FP4 MMAs.  An approximation of the bf16
    operand: fp32 out within 1e-3 of RMS of the exact linear (the oracle),
    bf16 out within the bf16 tolerance; per-row weight_scale_2 and a scalar
    input_scale."""
    import nvfp4
    from nvfp4 import synthetic

    wd = synthetic.linear_weights(N, K, seed=300 + K + N + M)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=M + 11))
    lin = nvfp4.NvFp4Linear(K, N, input_scale=0.5, weight_scale_2_rows=dev(wd["ws2"]))
    W, SF, X = dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16)
    flags = nvfp4._lib.FLAG_DIGIT_GEMV
    y32 = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_forward(lin, W, SF, X, y32, M, flags=flags)
    ybf = nvfp4.nvfp4_linear(lin, W, SF, X, flags=flags)
    torch.cuda.synchronize()
    assert nvfp4._lib.load().nvfp4_device_status() == 0
    ref = O.linear(wd["w"], wd["sf"], x, input_scale=0.5, ws2_rows=wd["ws2"])
    assert not torch.isnan(y32).any()
    assert rel_err(y32.cpu().numpy(), ref) <= DIGIT_TOL
    assert rel_err(ybf.float().cpu().numpy(), ref) <= TOL_BF16


def test_digit_gemv_repeatable_and_outliers(O, cuda):
    """Bitwise equal over repeated calls; a token with an outlier channel,
    an all-zero token and a tiny-magnitude token stay within tolerance."""
    import nvfp4
    from nvfp4 import synthetic

    N, K, M = 1536, 2048, 4
    wd = synthetic.linear_weights(N, K, seed=77)
    x = synthetic.activations(M, K, seed=78)
    x[0, 5] = 900.0
    x[1] = 0.0
    x[2] *= 1e-20
    x = synthetic.bf16_round(x)
    lin = nvfp4.NvFp4Linear(K, N, weight_scale_2_rows=dev(wd["ws2"]))
    W, SF, X = dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16)
    outs = []
    for _ in range(6):
        y = torch.empty((M, N), dtype=torch.float32, device=cuda)
        nvfp4.nvfp4_linear_forward(lin, W, SF, X, y, M, flags=nvfp4._lib.FLAG_DIGIT_GEMV)
        outs.append(y)
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    got = outs[0].cpu().numpy()
    ref = O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"])
    assert np.all(got[1] == 0.0)
    for t in (0, 2, 3):
        assert rel_err(got[t], ref[t]) <= DIGIT_TOL, t
