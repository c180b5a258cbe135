"""W4A4 mode on the GPU against the oracle, through the C ABI.

Quantizer (nvfp4_quantize_act): codes and blockscales bit-exact, including
round-to-nearest-even ties on the E2M1 grid, saturation, zero and tiny
groups.  GEMM (nvfp4_linear_w4a4, block-scaled FP4 tensor cores): every
product of two NVFP4 values is exact in fp32, so fp32 outputs match the
oracle to summation order (max|err| <= 1e-4 * RMS); bf16 outputs per element
within 2e-2 * RMS + 2^-8 * |ref| (the bf16-operand bound plus the output's own
rounding, half an ulp of bf16 being up to 2^-8 of the value).  nvfp4_linear_forward with
NVFP4_FLAG_W4A4 (stream-ordered scratch) equals the two-call form bitwise.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.sqrt(np.mean(ref * ref)))


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_quantize_act_bit_exact(O, cuda, dt):
    import nvfp4
    from nvfp4 import synthetic

    M, K = 37, 512
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=5) * 3.0)
    ins = float(np.abs(x).max() / (6 * 448))
    q, s = nvfp4.quantize_act(dev(x, dt), ins)
    rq, rs = O.quantize_act(x, ins)
    q, s = q.cpu().numpy(), s.cpu().numpy()
    assert np.array_equal(s, rs), np.argwhere(s != rs)[:5]
    assert np.array_equal(q, rq), np.argwhere(q != rq)[:5]


def test_quantize_act_ties_saturation_zero(O, cuda):
    import nvfp4

    # input_scale 1 and a group maximum of 6 give blockscale 1.0 exactly, so
    # the listed values sit exactly between E2M1 neighbours (ties to even).
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0,
                     -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0], np.float32)
    sat = np.array([7.0, -6.9, 0.1, 0.3] + [0.0] * 12, np.float32)  # scale 7/6 rounds down
    zero = np.zeros(16, np.float32)
    tiny = np.full(16, 1e-30, np.float32)
    huge = np.linspace(-1e6, 1e6, 16).astype(np.float32)
    x = np.concatenate([ties, sat, zero, tiny, huge, ties * 0.5])[None, :]
    x = np.concatenate([x, -x], axis=0)
    for ins in (1.0, 0.37):
        q, s = nvfp4.quantize_act(dev(x), ins)
        rq, rs = O.quantize_act(x, ins)
        assert np.array_equal(q.cpu().numpy(), rq), ins
        assert np.array_equal(s.cpu().numpy(), rs), ins


@pytest.mark.parametrize("N,K,M", [(256, 512, 1), (256, 512, 37), (384, 1024, 128),
                                   (200, 768, 300), (128, 256, 129)])
def test_w4a4_gemm_matches_oracle(O, cuda, N, K, M):
    import nvfp4
    from nvfp4 import synthetic

    wd = synthetic.linear_weights(N, K, seed=N + K + M)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=M + 1))
    ins = float(np.abs(x).max() / (6 * 448))
    lin = nvfp4.NvFp4Linear(K, N, input_scale=ins, weight_scale_2_rows=dev(wd["ws2"]))
    W, SF = dev(wd["w"]), dev(wd["sf"])
    q, s = nvfp4.quantize_act(dev(x, torch.bfloat16), ins)
    y32 = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    nvfp4.nvfp4_linear_w4a4(lin, W, SF, q, s, y32)
    ref = O.linear_w4a4(wd["w"], wd["sf"], x, ins, ws2_rows=wd["ws2"], n_threads=8)
    assert not torch.isnan(y32).any()
    assert rel_err(y32.cpu().numpy(), ref) <= 1e-4
    ybf = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    nvfp4.nvfp4_linear_w4a4(lin, W, SF, q, s, ybf)
    rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    excess = np.abs(ybf.float().cpu().numpy() - ref) - (TOL_BF16 * rms + 2.0 ** -8 * np.abs(ref))
    assert excess.max() <= 0.0
    # The flag form quantizes into stream-ordered scratch: bitwise the same.
    yf = nvfp4.nvfp4_linear(lin, W, SF, dev(x, torch.bfloat16), out_dtype=torch.float32,
                            flags=nvfp4._lib.FLAG_W4A4)
    assert torch.equal(yf, y32)


def test_w4a4_prefill_config2_sampled(O, cuda):
    """Prefill shape: x [512, 4096], W [14336, 4096], input_scale =
    max|x| / (6 * 448); oracle on a sample of rows and output features."""
    import nvfp4
    from nvfp4 import synthetic

    M, K, N = 512, 4096, 14336
    wd = synthetic.linear_weights(N, K, seed=77)
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=78))
    ins = float(np.abs(x).max() / (6 * 448))
    lin = nvfp4.NvFp4Linear(K, N, input_scale=ins, weight_scale_2_rows=dev(wd["ws2"]))
    y = nvfp4.nvfp4_linear(lin, dev(wd["w"]), dev(wd["sf"]), dev(x, torch.bfloat16),
                           out_dtype=torch.float32, flags=nvfp4._lib.FLAG_W4A4)
    rows = np.sort(np.random.default_rng(1).choice(M, 24, replace=False))
    cols = np.sort(np.random.default_rng(2).choice(N, 384, replace=False))
    ref = O.linear_w4a4(wd["w"], wd["sf"], x, ins, ws2_rows=wd["ws2"], rows=rows, cols=cols,
                        n_threads=8)
    got = y.cpu().numpy()[np.ix_(rows, cols)]
    assert rel_err(got, ref) <= 1e-4


def test_w4a4_repeatable(cuda):
    """Ten W4A4 GEMMs at M = 512, K = 4096, N = 14336 are bitwise identical
    (the scale factors staged by TMA are read before the stage is refilled)."""
    import nvfp4
    from nvfp4 import synthetic

    M, K, N = 512, 4096, 14336
    wd = synthetic.linear_weights_cuda(N, K, seed=91)
    x = torch.randn((M, K), device=cuda).to(torch.bfloat16)
    ins = float(x.float().abs().max().item() / (6 * 448))
    lin = nvfp4.NvFp4Linear(K, N, input_scale=ins, weight_scale_2_rows=wd["ws2"])
    first = None
    for i in range(10):
        y = nvfp4.nvfp4_linear(lin, wd["w"], wd["sf"], x, out_dtype=torch.float32,
                               flags=nvfp4._lib.FLAG_W4A4)
        if first is None:
            first = y
            assert not torch.isnan(first).any()
        else:
            assert torch.equal(y, first), f"call {i} differs"
