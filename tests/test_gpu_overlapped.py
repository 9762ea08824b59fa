"""Context::gemm for Scheme II INT8 with the GEMM overlapping A's upload (calls of at least 4096 rows).

The pipeline starts on a plan made from B's statistics and A's first band of rows and is confirmed, or
run again, with the reference's plan from the complete statistics; nothing is written to C before every
value is checked. The result must be the device pipeline's under the reference's plan, bit for bit, in
either case; an invalid value in A's last band must leave C untouched; and C may alias A.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu



def _opts(oztt, **kw):
    return oztt.Options(format=oztt.Format.INT8, **kw)


def test_overlapped_equals_device_pipeline(oztt, oracle, cuda):
    m, n, k = 4224, 1000, 700
    a, b = oracle.gen_inputs(m, n, k, 0.5, 21)
    c = np.empty(m * n)
    info = oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt))
    ph = oztt.ii_int8_last_phases()
    assert ph["bands"] >= 2 and ph["replanned"] == 0
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    assert (info.moduli, info.integer_bits, info.reconstruction_passes) == (plan.S, plan.b, 2 if plan.two_pass else 1)
    want = oztt.ii_int8_run(a, b, m, n, k, plan)
    assert np.array_equal(c.view(np.uint64), want.view(np.uint64))


def test_replanned_when_the_first_band_misleads(oztt, oracle, cuda):
    """A's first band has a narrow range of magnitudes and the rest a wide one: the first plan's width
    differs from the reference's, the pipeline runs again, and C is the reference plan's."""
    m, n, k = 4224, 512, 640
    a, b = oracle.gen_inputs(m, n, k, 0.0, 22)
    A = a.reshape(m, k)
    rng = np.random.default_rng(5)
    A[2304:] *= np.exp2(rng.integers(-40, 40, (m - 2304, k)))  # beyond the first band (2176 rows)
    c = np.empty(m * n)
    oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt))
    ph = oztt.ii_int8_last_phases()
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    want = oztt.ii_int8_run(a, b, m, n, k, plan)
    assert np.array_equal(c.view(np.uint64), want.view(np.uint64))
    assert ph["replanned"] == 1, "the first band was expected to give another plan"


def test_invalid_value_in_the_last_band_leaves_c_untouched(oztt, oracle, cuda):
    m, n, k = 4224, 300, 200
    a, b = oracle.gen_inputs(m, n, k, 0.5, 23)
    a[(m - 1) * k + 5] = np.inf
    c = np.full(m * n, 123.0)
    with pytest.raises(ValueError, match="A contains NaN or infinity"):
        oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt))
    assert np.all(c == 123.0)


def test_c_may_alias_a(oztt, oracle, cuda):
    m = n = k = 4096
    a, b = oracle.gen_inputs(m, n, k, 0.5, 24)
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    want = oztt.ii_int8_run(a, b, m, n, k, plan)
    oztt.Context().gemm(a, b, a, m, n, k, _opts(oztt))  # C written over A
    assert np.array_equal(a.view(np.uint64), want.view(np.uint64))
