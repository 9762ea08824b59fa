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
