"""The certified plan decision of the overlapped Context::gemm path (host logic, CPU).

The path measures A's rows with one fast pass (maxima exact; sums of squares and sketch values in FP64 in a
warp's order, with the sums of |terms|) and bounds the reference's statistics from them, so that the
reference's width cap and number of passes are decided without its sequential long-double sums. Here the
pass is restated in numpy on seeded inputs and the bounds are checked against the reference's exact values
(the host planner's statistics, equal to the reference's): they must contain nA and nC, and a decided plan
must take the reference's decisions.
"""

import ctypes

import numpy as np
import pytest

VECTORS = 8


def _b_parts(oztt, b, k, n):
    """B's exact parts as the reference computes them: column maxima, scale, scaled column sums of squares
    (sequential), and the sketch y_l = B g_l in long double, rounded to double."""
    B = b.reshape(k, n)
    cmax = np.abs(B).max(axis=0)
    top = cmax.max()
    _, e = np.frexp(top)
    rgB = float(np.ldexp(1.0, -int(min(max(e, -1000), 1000)))) if top > 0 else 1.0
    w = B * rgB
    cs2 = np.cumsum(w * w, axis=0)[-1]
    N = (n + 63) // 64 * 64
    g = oztt.policy_vectors(N)[:, :n]
    y = np.empty((VECTORS, k))
    xs = w.astype(np.longdouble)
    for l in range(VECTORS):
        prods = xs * g[l].astype(np.longdouble)[None, :]
        y[l] = np.cumsum(prods, axis=1)[:, -1].astype(np.float64)
    return cmax, cs2, rgB, y


def _cert_rows(a, m, k, y):
    A = a.reshape(m, k)
    out = np.zeros((m, 18))
    out[:, 0] = np.abs(A).max(axis=1)
    out[:, 1] = (A * A).sum(axis=1)
    t = A[:, None, :] * y[None, :, :]  # m x 8 x k
    out[:, 2:10] = t.sum(axis=2)
    out[:, 10:18] = np.abs(t).sum(axis=2)
    return out


@pytest.mark.parametrize("m,n,k,phi,seed", [(96, 80, 120, 0.5, 1), (130, 70, 200, 2.0, 2), (64, 64, 300, 4.0, 3),
                                            (200, 50, 64, -1.0, 4), (77, 99, 150, 1.0, 5)])
@pytest.mark.parametrize("recon", [0, 1, 2])
def test_bounds_contain_the_reference_and_decide_as_it(oztt, oracle, m, n, k, phi, seed, recon):
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    exact = oztt.ii_int8_plan(a, b, m, n, k, reconstruction=recon)
    cmax, cs2, rgB, y = _b_parts(oztt, b, k, n)
    cert = np.ascontiguousarray(_cert_rows(a, m, k, y))
    plan = oztt.IIPlan()
    decided = ctypes.c_int32()
    bounds = np.zeros(4)
    oztt.call("oztt_test_certified_plan", cert.ctypes.data, m, n, k, np.ascontiguousarray(cmax).ctypes.data,
              np.ascontiguousarray(cs2).ctypes.data, rgB, 0, recon, ctypes.byref(plan), ctypes.byref(decided),
              bounds.ctypes.data)
    assert bounds[0] <= exact.nA <= bounds[1], (bounds[:2], exact.nA)
    assert bounds[2] <= exact.nC <= bounds[3], (bounds[2:], exact.nC)
    assert (bounds[1] - bounds[0]) <= 1e-9 * exact.nA and (bounds[3] - bounds[2]) <= 1e-9 * exact.nC
    assert decided.value == 1
    assert (plan.S, plan.b, plan.b_cap, plan.two_pass, plan.moduli_list) == \
           (exact.S, exact.b, exact.b_cap, exact.two_pass, exact.moduli_list)
