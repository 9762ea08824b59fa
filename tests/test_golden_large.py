"""The oracle against the reference device's published outputs at n = 3520 (tools/validated/all.csv:12-13).

The evaluator's table suite (evaluation/evaluate.cpp:162-180, numerics.hpp:19-38): mt19937 seed 7,
uniform(-1, 1), Scheme II INT8 with max_moduli 16, one pass and b = 54; Scheme I INT8 with 8 slices.
The oracle's scaling, slicing and reconstruction run as they are; the integer products (exact: every
partial sum is an integer below 2^53) go through float64 matrix products so that the case finishes in
seconds. Matching the published FNV hash means every output bit equals the reference device's.
"""

import numpy as np
import pytest

from oracle_lib import pad, round_up

N = 3520
PUBLISHED = {"II": "a7bb9bd6f452e753", "I": "3ec48d5faecdf98f"}


@pytest.fixture(scope="module")
def inputs(oracle):
    a, b = oracle.gen_inputs(N, N, N, -1.0, 7)
    M, K = round_up(N, 64), round_up(N, 32)
    return pad(a, N, N, M, K), pad(b, N, N, K, M), M


def test_scheme_ii_3520(oracle, inputs):
    ap, bp, M = inputs
    rc, plan, err = oracle.plan(ap, bp, M, M, M, 16, 1, 54)
    assert rc == 0, err
    assert (plan.S, plan.b) == (16, 54)
    _, dA, _ = oracle.scale(ap, M, M, 0, plan.shift)
    _, dB, _ = oracle.scale(bp, M, M, 1, plan.shift)
    ra = oracle.split(ap, M, M, 0, dA, plan).reshape(plan.S, M, M)
    rb = oracle.split(bp, M, M, 1, dB, plan).reshape(plan.S, M, M)
    cs = np.empty((plan.S, M, M), dtype=np.int32)
    for s in range(plan.S):
        cs[s] = (ra[s].astype(np.float64) @ rb[s].astype(np.float64).T).astype(np.int32)
    c = oracle.recon(cs.reshape(-1), M, M, dA, dB, plan, exact=False).reshape(M, M)[:N, :N]
    assert oracle.output_hash(np.ascontiguousarray(c).reshape(-1)) == PUBLISHED["II"]


def test_scheme_i_3520(oracle, inputs):
    ap, bp, M = inputs
    p = 8
    _, dA, _ = oracle.scale(ap, M, M, 0, -1)
    _, dB, _ = oracle.scale(bp, M, M, 1, -1)
    sa = oracle.i_slice(ap, M, M, 0, dA, p).reshape(p, M, M).astype(np.float64)
    sb = oracle.i_slice(bp, M, M, 1, dB, p).reshape(p, M, M).astype(np.float64)
    pd = np.zeros((p, M, M))
    for d in range(p):
        for i in range(d + 1):
            pd[d] += sa[i] @ sb[d - i].T
    c = oracle.i_recon(pd.astype(np.int32).reshape(-1), p, M, M, dA, dB, exact=False).reshape(M, M)[:N, :N]
    assert oracle.output_hash(np.ascontiguousarray(c).reshape(-1)) == PUBLISHED["I"]
