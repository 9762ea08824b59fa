"""The certified plan decision of the overlapped Context::gemm path (host logic, CPU).

The path measures B's rows (sketch sums, sums of |terms| and of squares in FP64, its column maxima exactly) and
A's rows (maxima exact; sums of squares and sketch values in FP64 in a warp's order, with the sums of |terms|)
with fast passes and bounds the reference's statistics from them, so that the reference's width cap and
number of passes are decided without its sequential long-double sums. Here the passes are restated in numpy
on seeded inputs and the bounds are checked against the reference's exact values (the host planner's
statistics, equal to the reference's): they must contain nA, nB and nC, and a decided plan must take the
reference's decisions -- with B's exact sketch, and with B's bounded one.
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


def _b_bounded(oztt, b, k, n):
    """B's bounded pass restated: per row of B the FP64 sums of b g_l, |b g_l| and b^2 (numpy's order, within
    the pass's error bound), the exact column maxima and scale; the scaled sketch, the bound ew of its error
    against the reference's, and the bounds of nB."""
    B = b.reshape(k, n)
    cmax = np.abs(B).max(axis=0)
    top = cmax.max()
    _, e = np.frexp(top)
    rgB = float(np.ldexp(1.0, -int(min(max(e, -1000), 1000)))) if top > 0 else 1.0
    N = (n + 63) // 64 * 64
    g = oztt.policy_vectors(N)[:, :n]
    acc = np.zeros((k, 17))
    t = B[:, None, :] * g[None, :, :]  # k x 8 x n
    acc[:, 0:8] = t.sum(axis=2)
    acc[:, 8:16] = np.abs(t).sum(axis=2)
    acc[:, 16] = (B * B).sum(axis=1)
    acc = np.ascontiguousarray(acc)
    out3 = np.zeros(3)
    oztt.call("oztt_test_bounded_nb", acc.ctypes.data, k, n, rgB, out3.ctypes.data)
    c1 = out3[2]
    y = (acc[:, 0:8] * rgB).T.copy()  # 8 x k
    ew = (c1 * (acc[:, 8:16] * rgB) + 2.0 ** -53 * np.abs(acc[:, 0:8] * rgB)).max(axis=1)
    return cmax, rgB, y, ew, out3[0], out3[1]


def _cert_rows(a, m, k, y, ew=None):
    A = a.reshape(m, k)
    out = np.zeros((m, 19))
    out[:, 0] = np.abs(A).max(axis=1)
    out[:, 1] = (A * A).sum(axis=1)
    t = A[:, None, :] * y[None, :, :]  # m x 8 x k
    out[:, 2:10] = t.sum(axis=2)
    out[:, 10:18] = np.abs(t).sum(axis=2)
    if ew is not None:
        out[:, 18] = np.abs(A) @ ew
    return np.ascontiguousarray(out)


def _certified(oztt, cert, m, n, k, cmax, nb_lo, nb_hi, rgB, recon):
    plan = oztt.IIPlan()
    decided = ctypes.c_int32()
    bounds = np.zeros(6)
    oztt.call("oztt_test_certified_plan", cert.ctypes.data, m, n, k, np.ascontiguousarray(cmax).ctypes.data,
              nb_lo, nb_hi, rgB, 0, recon, ctypes.byref(plan), ctypes.byref(decided), bounds.ctypes.data)
    return plan, decided.value, bounds


@pytest.mark.parametrize("m,n,k,phi,seed", [(96, 80, 120, 0.5, 1), (130, 70, 200, 2.0, 2), (64, 64, 300, 4.0, 3),
                                            (200, 50, 64, -1.0, 4), (77, 99, 150, 1.0, 5)])
@pytest.mark.parametrize("recon", [0, 1, 2])
def test_bounds_contain_the_reference_and_decide_as_it(oztt, oracle, m, n, k, phi, seed, recon):
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    exact = oztt.ii_int8_plan(a, b, m, n, k, reconstruction=recon)
    cmax, cs2, rgB, y = _b_parts(oztt, b, k, n)
    nb = float(np.cumsum(cs2)[-1])  # the reference's sum over the columns, in order
    plan, decided, bounds = _certified(oztt, _cert_rows(a, m, k, y), m, n, k, cmax, nb, nb, rgB, recon)
    assert bounds[0] <= exact.nA <= bounds[1], (bounds[:2], exact.nA)
    assert bounds[2] <= exact.nC <= bounds[3], (bounds[2:4], exact.nC)
    assert (bounds[1] - bounds[0]) <= 1e-9 * exact.nA and (bounds[3] - bounds[2]) <= 1e-9 * exact.nC
    assert decided == 1
    assert (plan.S, plan.b, plan.b_cap, plan.two_pass, plan.moduli_list) == \
           (exact.S, exact.b, exact.b_cap, exact.two_pass, exact.moduli_list)


@pytest.mark.parametrize("m,n,k,phi,seed", [(96, 80, 120, 0.5, 1), (130, 70, 200, 2.0, 2), (64, 64, 300, 4.0, 3),
                                            (200, 50, 64, -1.0, 4), (77, 99, 150, 1.0, 5), (50, 300, 90, 0.5, 6)])
@pytest.mark.parametrize("recon", [0, 1, 2])
def test_bounds_from_b_bounded_pass(oztt, oracle, m, n, k, phi, seed, recon):
    """B measured by the bounded pass (no long-double sums anywhere): the bounds still contain the
    reference's nA, nB and nC, stay tight, and decide as the reference."""
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    exact = oztt.ii_int8_plan(a, b, m, n, k, reconstruction=recon)
    cmax, rgB, y, ew, nb_lo, nb_hi = _b_bounded(oztt, b, k, n)
    plan, decided, bounds = _certified(oztt, _cert_rows(a, m, k, y, ew), m, n, k, cmax, nb_lo, nb_hi, rgB, recon)
    assert bounds[0] <= exact.nA <= bounds[1], (bounds[:2], exact.nA)
    assert bounds[2] <= exact.nC <= bounds[3], (bounds[2:4], exact.nC)
    assert bounds[4] <= exact.nB <= bounds[5], (bounds[4:], exact.nB)
    assert (bounds[3] - bounds[2]) <= 1e-6 * exact.nC and (bounds[5] - bounds[4]) <= 1e-9 * exact.nB
    assert decided == 1
    assert (plan.S, plan.b, plan.b_cap, plan.two_pass, plan.moduli_list) == \
           (exact.S, exact.b, exact.b_cap, exact.two_pass, exact.moduli_list)
