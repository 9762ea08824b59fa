"""Context::gemm for Scheme II INT8 computing while its operands upload (calls of at least 4096 rows).

The upload order is B's first block of columns, A's first part (half of its rows, whole bands of 1024), B's
next blocks, the rest of A, B's last blocks. The pipeline starts on a plan estimated from A's first part and B's first block and is
confirmed, or run again, with the reference's plan from the complete statistics; C is read back as its
pieces finish once every value is checked (unless C overlaps A or B, or some plan for the dimensions could
fail). The result must be the device
pipeline's under the reference's plan, bit for bit, in either case; an invalid value in A's last band, or a
plan that fails, must leave C untouched; and C may alias A.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu



def _opts(oztt, **kw):
    return oztt.Options(format=oztt.Format.INT8, **kw)


def test_overlapped_equals_device_pipeline(oztt, oracle, cuda):
    """phi = 1 puts log2 of the policy's k2 near 3.26 for the whole matrices and for the first parts (A's
    first 3072 rows, B's first 256 columns) alike, well inside one width: the first plan is confirmed."""
    m, n, k = 4224, 1000, 700
    a, b = oracle.gen_inputs(m, n, k, 1.0, 21)
    c = np.empty(m * n)
    info = oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt))
    ph = oztt.ii_int8_last_phases()
    assert ph["bands"] >= 2 and ph["replanned"] == 0 and ph["early_readback"] == 1
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    assert (info.moduli, info.integer_bits, info.reconstruction_passes) == (plan.S, plan.b, 2 if plan.two_pass else 1)
    want = oztt.ii_int8_run(a, b, m, n, k, plan)
    assert np.array_equal(c.view(np.uint64), want.view(np.uint64))


def test_replanned_when_the_first_part_misleads(oztt, oracle, cuda):
    """A's first part has a narrow range of magnitudes and the rest a wide one: the first plan's width
    (53 bits) differs from the reference's (56), the pipeline runs again after C's bands were read back on
    the first plan, and C is the reference plan's."""
    m, n, k = 4224, 512, 640
    a, b = oracle.gen_inputs(m, n, k, 0.0, 22)
    A = a.reshape(m, k)
    rng = np.random.default_rng(5)
    A[3072:] *= np.exp2(rng.integers(-40, 40, (m - 3072, k)))  # beyond the first part (3072 rows)
    c = np.empty(m * n)
    oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt))
    ph = oztt.ii_int8_last_phases()
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    want = oztt.ii_int8_run(a, b, m, n, k, plan)
    assert np.array_equal(c.view(np.uint64), want.view(np.uint64))
    assert ph["replanned"] == 1, "the first part was expected to give another plan"
    assert ph["early_readback"] == 1


def test_invalid_value_in_the_last_band_leaves_c_untouched(oztt, oracle, cuda):
    m, n, k = 4224, 300, 200
    a, b = oracle.gen_inputs(m, n, k, 0.5, 23)
    a[(m - 1) * k + 5] = np.inf
    c = np.full(m * n, 123.0)
    with pytest.raises(ValueError, match="A contains NaN or infinity"):
        oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt))
    assert np.all(c == 123.0)


@pytest.mark.parametrize("where,message", [("a_first_half", "A contains NaN or infinity"),
                                           ("b", "B contains NaN or infinity"),
                                           ("a_range", "each nonzero row maximum of A")])
def test_invalid_values_reported_in_order_and_c_untouched(oztt, oracle, cuda, where, message):
    """Invalid values in A's first part (its maxima measured on the device) or in B (on the host's threads):
    the front end's report, C never written."""
    m, n, k = 4224, 300, 200
    a, b = oracle.gen_inputs(m, n, k, 0.5, 26)
    if where == "a_first_half":
        a[10 * k + 3] = np.nan
    elif where == "b":
        b[(k - 1) * n + 7] = -np.inf
    else:
        a[20 * k: 21 * k] = 2.0 ** -140  # a row whose maximum is below 2^-126
    c = np.full(m * n, 5.0)
    with pytest.raises(ValueError, match=message):
        oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt))
    assert np.all(c == 5.0)


def test_failing_plan_leaves_c_untouched(oztt, oracle, cuda):
    """Eight moduli cannot cover 53 bits: no plan exists, the error is reported and C is not written."""
    m, n, k = 4224, 256, 512
    a, b = oracle.gen_inputs(m, n, k, 0.5, 25)
    c = np.full(m * n, 7.0)
    with pytest.raises(RuntimeError):
        oztt.Context().gemm(a, b, c, m, n, k, _opts(oztt, max_moduli=8))
    assert np.all(c == 7.0)


def test_c_may_alias_a(oztt, oracle, cuda):
    m = n = k = 4096
    a, b = oracle.gen_inputs(m, n, k, 0.5, 24)
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    want = oztt.ii_int8_run(a, b, m, n, k, plan)
    oztt.Context().gemm(a, b, a, m, n, k, _opts(oztt))  # C written over A
    assert oztt.ii_int8_last_phases()["early_readback"] == 0  # C only after A has landed
    assert np.array_equal(a.view(np.uint64), want.view(np.uint64))
