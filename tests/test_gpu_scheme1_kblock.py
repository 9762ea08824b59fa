"""Scheme I diagonal products in K blocks (FP8, BF16, FP16 and TF32 slices with a long K).

The diagonal sums are exact in the tensor cores' s32 accumulators while (L+1) K dmax^2 < 2^31; beyond that
the products run block by block over K and the int32 block sums are added in int64 before the exact
Horner evaluation (the reference sums FP32 partial products per K block, src/ozaki1.cpp:238-262). A test
hook caps the block length so that the blocked path runs at small sizes: its C must equal, bit for bit,
the unblocked path's and the oracle's exact restatement, through the device pipeline and through
Context::gemm.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture()
def kblock(oztt):
    yield lambda kb: oztt.lib.oztt_test_scheme1_kblock(kb)
    oztt.lib.oztt_test_scheme1_kblock(0)


@pytest.mark.parametrize("fmt,p", [(4, 7), (0, 6), (5, 5)])
@pytest.mark.parametrize("m,n,k", [(200, 150, 1000), (130, 300, 513)])
def test_blocked_equals_unblocked(oztt, oracle, cuda, kblock, fmt, p, m, n, k):
    a, b = oracle.gen_inputs(m, n, k, 1.0, 17)
    plan = oztt.i_int8_plan(a, b, m, n, k, slices=p, fmt=oztt.Format(fmt))
    want = oztt.i_int8_run(a, b, m, n, k, plan)
    exact = oracle.i_emulate(a, b, m, n, k, p, exact=True, fmt=fmt)
    assert np.array_equal(want.view(np.uint64), exact.view(np.uint64))
    for kb in (128, 256, 384):
        kblock(kb)
        got = oztt.i_int8_run(a, b, m, n, k, plan)
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), kb
        c = np.empty(m * n)
        oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(scheme=oztt.Scheme.I, format=oztt.Format(fmt), slices=p))
        assert np.array_equal(c.view(np.uint64), want.view(np.uint64)), kb
