"""The Scheme II INT8 planner: the library's decisions equal the reference's.

CPU only (the planner is host code in liboztt.so). Three-way agreement over the fixture table made
from the reference's own planner (tests/golden/make_golden.py): liboztt.so (product), the oracle's
restatement, and — where oracle/_ref exists — the reference compiled in place.
"""

import json
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle_lib import pad, round_up

GOLDEN = json.loads((Path(__file__).parent / "golden" / "ref_cases.json").read_text())


def product_selection(oztt, K, num_moduli, b_cap):
    """Moduli selection through the public planner seam: a 1 x K times K x 1 problem with a fixed width
    (the evaluator's fixed_bits) and one reconstruction pass, so no statistics are measured."""
    a = np.ones(K)
    b = np.ones(K)
    try:
        p = oztt.ii_int8_plan(a, b, 1, 1, K, max_moduli=num_moduli, reconstruction=1, fixed_bits=b_cap)
    except RuntimeError:
        return None
    return p


def test_moduli_table_product(oztt):
    bad = []
    for row in GOLDEN["moduli_table"]:
        p = product_selection(oztt, row["K"], row["num_moduli"], row["b_cap"])
        if not row["ok"]:
            if p is not None:
                bad.append((row, "accepted"))
            continue
        if p is None:
            bad.append((row, "rejected"))
            continue
        got = (p.S, p.b, p.moduli_list, [int(p.yi[i]) for i in range(p.S)])
        want = (row["S"], row["b"], row["moduli"], row["yi"])
        if got != want:
            bad.append((row, got))
    assert not bad, bad[:5]


def test_moduli_table_oracle(oracle):
    bad = []
    for row in GOLDEN["moduli_table"]:
        p = oracle.choose_moduli(row["K"], row["num_moduli"], row["b_cap"])
        got = (int(p.ok), int(p.acc_ok), p.S, p.b, p.m_cap, p.ncand, p.moduli)
        want = (row["ok"], row["acc_ok"], row["S"], row["b"], row["m_cap"], row["ncand"], row["moduli"])
        if got != want:
            bad.append((row, got))
    assert not bad, bad[:5]


def _hexs(vals):
    return [float.hex(float(v)) for v in vals]


@pytest.mark.parametrize("idx", range(0, len(GOLDEN["plans"]), 1))
def test_plan_product_and_oracle(oztt, oracle, idx):
    case = GOLDEN["plans"][idx]
    m, n, k = case["m"], case["n"], case["k"]
    a, b = oracle.gen_inputs(m, n, k, case["phi"], case["seed"])
    # product
    try:
        p = oztt.ii_int8_plan(a, b, m, n, k, case["max_moduli"], case["passes"], case["fixed_bits"])
        prc = 0
    except RuntimeError:
        p, prc = None, 1
    assert prc == case["rc"]
    if p is not None:
        assert (p.S, p.b, p.two_pass, p.moduli_list, p.b_cap) == (case["S"], case["b"], case["two_pass"],
                                                                  case["moduli"], case["b_cap"])
        assert _hexs((p.TA, p.TB, p.nA, p.nB, p.nC)) == case["stats"]
    # oracle restatement on the padded matrices
    M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
    rc, q, _ = oracle.plan(pad(a, m, k, M, K), pad(b, k, n, K, N), M, N, K, case["max_moduli"], case["passes"],
                           case["fixed_bits"])
    assert rc == case["rc"]
    assert (q.S, q.b, q.moduli) == (case["S"], case["b"], case["moduli"])
    if rc == 0:
        assert q.two_pass == case["two_pass"]
        assert _hexs((q.TA, q.TB, q.nA, q.nB, q.nC)) == case["stats"]


def test_plan_constants_match_oracle(oztt, oracle):
    """CRT constants passed to the kernels: y_i, fl32(1/m_i), 2^(20j) mod m_i, shift and digits."""
    for (K, num, bcap) in [(64, 16, 54), (4096, 24, 56), (16384, 16, 54), (14080, 16, 70), (256, 24, 81),
                           (1 << 20, 24, 54)]:
        p = product_selection(oztt, K, num, bcap)
        q = oracle.choose_moduli(K, num, bcap)
        assert p is not None and q.ok
        assert p.moduli_list == q.moduli and p.b == q.b and p.nd == q.nd and p.shift == q.shift
        for i in range(p.S):
            assert p.yi[i] == q.yi[i]
            assert struct.pack("f", p.rinv[i]) == struct.pack("f", q.rinv[i])
            for j in range(4):
                assert p.c[j][i] == q.c[j][i]


def test_reference_planner_live(oracle, ref_plan):
    """The oracle planner vs the reference planner compiled in place, on extra inputs."""
    for (m, n, k, phi, seed, mm, passes) in [(64, 64, 320, 3.0, 1, 0, 0), (100, 60, 50, 0.5, 2, 18, 0),
                                             (64, 128, 2048, -1.0, 3, 0, 2), (8, 8, 40000, 0.0, 4, 0, 0)]:
        a, b = oracle.gen_inputs(m, n, k, phi, seed)
        M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
        ap, bp = pad(a, m, k, M, K), pad(b, k, n, K, N)
        rc1, p1, _ = oracle.plan(ap, bp, M, N, K, mm, passes, 0)
        rc2, p2 = ref_plan.plan(ap, bp, M, N, K, mm, passes, 0)
        assert (rc1, p1.S, p1.b, p1.moduli, p1.two_pass) == (rc2, p2.S, p2.b, p2.moduli, p2.two_pass)
        assert _hexs((p1.TA, p1.TB, p1.nA, p1.nB, p1.nC)) == _hexs((p2.TA, p2.TB, p2.nA, p2.nB, p2.nC))
        for i in range(p1.S):
            assert (p1.yi[i], p1.W_hi, p1.W_lo, p1.qw, p1.nsmall0, p1.nsmall1, p1.nsmall2) == \
                   (p2.yi[i], p2.W_hi, p2.W_lo, p2.qw, p2.nsmall0, p2.nsmall1, p2.nsmall2)
            assert list(p1.rp0[i]) == list(p2.rp0[i]) and list(p1.rp1[i]) == list(p2.rp1[i])
            assert list(p1.rp2[i]) == list(p2.rp2[i])
