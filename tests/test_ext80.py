"""The 64-bit-significand arithmetic that the device uses to reproduce the reference's long double
sums (oztt_b200/csrc/ext80.h), against the host's own x87 long double through numpy.longdouble.

The reference forms acc += (long double)(x*rg) * g in estimate_product_norm
(src/backend/common/norm_estimate.hpp:48-73); the device sketch must give the same double for every row.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.skipif(np.finfo(np.longdouble).nmant != 63, reason="needs the x87 80-bit long double")


def reference_dot(x, g, rg):
    acc = np.longdouble(0)
    for xj, gj in zip(x, g):
        acc = acc + np.longdouble(xj * rg) * np.longdouble(gj)
    return float(acc)


@pytest.mark.parametrize("case", range(8))
def test_ext80_dot_matches_long_double(oztt, case):
    rng = np.random.default_rng(100 + case)
    n = [1, 7, 64, 257, 1000, 4096, 513, 2048][case]
    if case < 4:
        x = rng.uniform(-1, 1, n)
        g = rng.standard_normal(n)
    elif case == 4:  # wide exponent range, heavy cancellation
        x = rng.standard_normal(n) * np.exp2(rng.integers(-200, 200, n))
        g = rng.standard_normal(n)
    elif case == 5:  # terms that cancel exactly in pairs, then a tiny remainder
        x = np.repeat(rng.standard_normal(n // 2), 2)
        g = np.tile([1.0, -1.0], n // 2)
        x[-1] += 2.0 ** -60
    elif case == 6:  # subnormal and zero inputs, signed zeros
        x = rng.standard_normal(n) * 1e-310
        x[::5] = 0.0
        x[1::7] = -0.0
        g = rng.standard_normal(n)
    else:  # products that round at the 64-bit boundary: significands full of ones
        x = 1.0 - np.exp2(-rng.integers(1, 53, n).astype(float))
        g = (1.0 + np.exp2(-rng.integers(1, 53, n).astype(float))) * np.where(rng.random(n) < 0.5, -1, 1)
    rg = float(np.exp2(-rng.integers(0, 4)))
    got = oztt.lib.oztt_test_ext80_dot(x.ctypes.data, g.ctypes.data, n, rg)
    want = reference_dot(x, g, rg)
    assert np.float64(got).view(np.uint64) == np.float64(want).view(np.uint64)


def _mixed_case(seed, n=1500):
    """Sums whose additions hit every alignment of the 64-bit window: exponent gaps around 0, 64 and
    128 and beyond, carries out of the top bit, exact and near cancellations, full significands."""
    rng = np.random.default_rng(1000 + seed)
    style = seed % 4
    sign = np.where(rng.random(n) < 0.5, -1.0, 1.0)
    frac = 1.0 + rng.integers(0, 2 ** 52, n) * 2.0 ** -52
    if style == 0:  # exponent gaps spread over [0, 160]
        x = sign * frac * np.exp2(rng.integers(-80, 81, n).astype(float))
        g = frac[::-1] * np.exp2(rng.integers(-80, 81, n).astype(float))
    elif style == 1:  # gaps clustered at 63, 64, 65 and 127, 128, 129 bits
        gap = rng.choice([0, 1, 62, 63, 64, 65, 66, 126, 127, 128, 129, 130], n).astype(float)
        x = sign * frac * np.exp2(-gap)
        g = 1.0 + rng.integers(0, 2 ** 52, n) * 2.0 ** -52
    elif style == 2:  # near cancellations: each term undoes most of the previous one
        base = rng.standard_normal(n)
        x = base.copy()
        x[1::2] = -base[:-1:2] * (1.0 + np.exp2(-rng.integers(1, 70, n // 2).astype(float)))
        g = np.ones(n)
    else:  # significands full of ones, products rounding at the 64-bit boundary, mixed signs
        x = sign * (2.0 - np.exp2(-rng.integers(40, 53, n).astype(float)))
        g = (2.0 - np.exp2(-rng.integers(1, 53, n).astype(float))) * np.exp2(rng.integers(-70, 71, n).astype(float))
    return x, g


@pytest.mark.parametrize("seed", range(16))
def test_ext80_dot_mixed_alignments(oztt, seed):
    x, g = _mixed_case(seed)
    got = oztt.lib.oztt_test_ext80_dot(x.ctypes.data, g.ctypes.data, len(x), 1.0)
    want = reference_dot(x, g, 1.0)
    assert np.float64(got).view(np.uint64) == np.float64(want).view(np.uint64), seed
