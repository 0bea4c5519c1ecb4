"""The power-of-two fast path of pass 1 rests on one fact: for a scale
inverse inv = 2^k, fp32(h) * inv is exact for every finite FP16 h when
-125 <= k <= 112 (every FP16 value is a multiple of 2^-24 and at most
65504 = (2 - 2^-10) * 2^15), so
the sum of squared unscaled gradients is inv^2 times the sum of the exact
h^2.  The kernel takes the fast path only for -102 <= k <= 111 (products
that stay normal f32 numbers), inside that range; any other scale goes
through the general path, which rounds in f32 as the reference does.
Checked exhaustively over all finite halves at the ends of both ranges, and
shown to fail just outside the exact one."""
import numpy as np


def finite_halves():
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    h = bits.view(np.float16)
    return h[np.isfinite(h)].astype(np.float32)


def exact_in_f32(h32, k):
    inv = np.float32(2.0 ** k)
    with np.errstate(over="ignore", under="ignore"):
        prod32 = (h32 * inv).astype(np.float64)   # f32 multiply, RNE, no FTZ
    exact = h32.astype(np.float64) * 2.0 ** k      # exact in double
    return np.array_equal(prod32, exact)


def test_products_exact_over_the_fast_path_range():
    h32 = finite_halves()
    for k in (-125, -103, -102, -101, -24, -16, 0, 16, 111, 112):
        assert exact_in_f32(h32, k), k


def test_products_inexact_just_outside():
    h32 = finite_halves()
    assert not exact_in_f32(h32, -126)             # the smallest subnormal halves round
    assert not exact_in_f32(h32, 113)              # 65504 * 2^113 overflows f32
