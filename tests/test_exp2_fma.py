"""Host model of the prefill kernel's FMA-pipe 2^x (exp2_fma_x2 in
tvp_prefill.cu), replayed in float32 with numpy: range reduction by the
1.5 * 2^23 addition, the cubic for 2^f, the exponent by an integer add.
Its relative error must stay far below a BF16 probability's rounding (2^-9)
over the kernel's range of exponents (masked keys are -inf, the lazy running
max lets arguments reach +8)."""
import numpy as np

C = np.array([0.99992806, 0.69326097, 0.24261113, 0.055171769], dtype=np.float32)
MAGIC = np.float32(12582912.0)


def exp2_fma(x):
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-125.0))
    t = (x + MAGIC).astype(np.float32)
    i = (t - MAGIC).astype(np.float32)
    f = (x - i).astype(np.float32)
    y = (C[3] * f + C[2]).astype(np.float32)
    y = (y * f + C[1]).astype(np.float32)
    y = (y * f + C[0]).astype(np.float32)
    bits = (y.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_over_the_kernel_range():
    x = np.linspace(-124.0, 10.0, 2_000_001, dtype=np.float32)
    got = exp2_fma(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    assert np.abs(got / want - 1).max() < 1e-4


def test_masked_and_very_small_arguments_give_a_tiny_normal():
    out = exp2_fma(np.array([-np.inf, -1000.0, -126.0, -125.0], dtype=np.float32))
    assert np.all(out > 0) and np.all(out < 1e-37)
    assert np.all(np.isfinite(out))


def test_integers_are_exact_powers_of_two_to_the_polynomial_error():
    x = np.arange(-120, 11, dtype=np.float32)
    assert np.abs(exp2_fma(x) / np.exp2(x.astype(np.float64)) - 1).max() < 1e-4
