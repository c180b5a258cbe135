"""The FP4-digit decomposition (oracle.fp4_digits) that the next decode GEMV
is planned around: bf16 activations written as a sum of D NVFP4 rows with
per-(token, digit) fp32 scales.  Pins its accuracy on CPU: how closely D
digits rebuild x, and the GEMV error against the exact W4A16 linear."""
import numpy as np
import pytest


def test_one_digit_is_the_w4a4_quantization(O):
    from nvfp4 import synthetic

    x = synthetic.bf16_round(synthetic.activations(3, 512, seed=4))
    codes, scs, sd = O.fp4_digits(x, digits=1)
    for t in range(3):
        s = np.float32(np.abs(x[t]).max()) / np.float32(6 * 448)
        assert sd[t] == s
        q, sc = O.quantize_act(x[t:t + 1], float(s))
        assert np.array_equal(codes[t], q[0]) and np.array_equal(scs[t], sc[0])


@pytest.mark.parametrize("digits,bound", [(2, 3e-2), (3, 3e-3), (4, 5e-4)])
def test_digits_rebuild_the_activations(O, digits, bound):
    """Each digit shrinks the residual about tenfold (measured 1.6e-2,
    1.4e-3, 1.4e-4 for 2, 3, 4 digits); errors are
    relative to the token's max |x|."""
    from nvfp4 import synthetic

    x = synthetic.bf16_round(synthetic.activations(8, 1024, seed=9) * 3.0)
    x[2, 7] = 400.0  # an outlier channel
    codes, scs, sd = O.fp4_digits(x, digits=digits)
    xh = O.fp4_digits_value(codes, scs, sd, digits=digits)
    err = np.abs(xh - x).max(axis=1) / np.abs(x).max(axis=1)
    assert err.max() <= bound, err


def test_digit_gemv_error_against_w4a16(O):
    """D = 4: the linear on the rebuilt activations is within 1e-3 of RMS of
    the linear on x (the tolerance of the GEMV parity tests is 2e-2)."""
    from nvfp4 import synthetic

    N, K, M = 256, 1024, 8
    wd = synthetic.moe_weights(1, K, N // 2, seed=3)
    w, sf = wd["gu_w"][0], wd["gu_sf"][0]
    x = synthetic.bf16_round(synthetic.activations(M, K, seed=5))
    ref = O.linear(w, sf, x)
    codes, scs, sd = O.fp4_digits(x, digits=4)
    got = O.linear(w, sf, O.fp4_digits_value(codes, scs, sd, digits=4))
    rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    assert np.abs(got - ref).max() / rms <= 1e-3
