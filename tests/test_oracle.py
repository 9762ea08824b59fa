"""The oracle pinned against the reference: its published device output and its own host code.

CPU only. These tests establish that oracle/liboz2oracle.so is a faithful restatement of the
reference's Scheme II INT8 path before the GPU tests use it as the checker.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle_lib import pad, round_up

GOLDEN = json.loads((Path(__file__).parent / "golden" / "ref_cases.json").read_text())


def test_published_device_hash(oracle):
    """tools/validated/quick.csv:13: n=128, seed 7, uniform, b=54, one pass -> fe063f5214e93e2e."""
    pub = GOLDEN["published"]
    n = pub["n"]
    a, b = oracle.gen_inputs(n, n, n, pub["phi"], pub["seed"])
    rc, c, plan, err = oracle.emulate(a, b, n, n, n, fixed_bits=pub["fixed_bits"], passes=0)
    assert rc == 0, err
    assert plan.S == pub["moduli"] and plan.b == pub["fixed_bits"] and plan.two_pass == 0
    assert oracle.output_hash(c) == pub["output_hash"]
    hi, lo = oracle.dot2(a, b, n, n, n)
    rel, ebits = oracle.accuracy(c, hi, lo)
    assert f"{rel:.11e}" == f"{pub['relative_fro']:.11e}"
    assert abs(ebits - pub["effective_bits"]) < 1e-9


@pytest.mark.parametrize("case", GOLDEN["emulations"], ids=lambda c: f"n{c['n']}-phi{c['phi']}-b{c['fixed_bits']}-"
                                                                    f"p{c['two_pass'] + 1}")
def test_oracle_matches_reference_emulation(oracle, case):
    """Output hashes of the reference's own host emulation (fixtures made by tests/golden/make_golden.py)."""
    n = case["n"]
    a, b = oracle.gen_inputs(n, n, n, case["phi"], case["seed"])
    rc, c, plan, err = oracle.emulate(a, b, n, n, n, max_moduli=case["num_moduli"], passes=2 if case["two_pass"] else 1,
                                      fixed_bits=case["fixed_bits"])
    assert rc == 0, err
    assert plan.moduli == case["moduli"]
    assert oracle.output_hash(c) == case["output_hash"]


def test_oracle_matches_reference_live(oracle, ref_emu):
    """Non-square, padded shapes against the reference's emulation compiled in place (when present)."""
    for (m, n, k, phi, seed, bfix, two) in [(70, 130, 90, -1.0, 2, 54, False), (64, 192, 64, 0.5, 4, 57, True),
                                            (128, 64, 300, 1.0, 8, 63, False)]:
        a, b = oracle.gen_inputs(m, n, k, phi, seed)
        M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
        ap, bp = pad(a, m, k, M, K), pad(b, k, n, K, N)
        s, cref, mods = ref_emu.emulate(ap, bp, M, N, K, bfix, 16, two)
        assert s > 0
        rc, c, plan, err = oracle.emulate(a, b, m, n, k, max_moduli=16, passes=2 if two else 1, fixed_bits=bfix)
        assert rc == 0, err
        assert plan.moduli == mods
        cref = cref.reshape(M, N)[:m, :n].reshape(-1)
        assert np.array_equal(c.view(np.uint64), cref.view(np.uint64))


def test_digit_error_bound(oracle):
    """|A' - X| <= 1 for the integer carried by the digits (digits.h:35-52), X = x * 2^(b-e)."""
    rng = np.random.default_rng(5)
    nd, b = 3, 54
    shift = b - 20 * (nd - 1)
    for _ in range(2000):
        x = float(rng.uniform(-1, 1) * 2.0 ** rng.integers(-60, 1))
        e = 1  # row maximum rounded up to 2^1 > |x|
        dg = oracle.digits(x, shift - e, nd).astype(np.float64)
        aprime = sum(int(d) * 2 ** (20 * (nd - 1 - i)) for i, d in enumerate(dg))
        X = x * 2.0 ** (b - e)
        assert abs(aprime - X) <= 1.0


def test_exact_recon_within_reference_tolerance(oracle):
    """The B200 exact CRT (restated in the oracle) vs the reference's triple-float CRT, componentwise:
    |C_exact - C_ref| <= 2^-65 * KM * 2^(2 shift - dA_i - dB_j) + 2 ulp(C_ref) for one pass."""
    for (n, phi, seed) in [(64, -1.0, 1), (96, 0.5, 2), (64, 2.0, 3)]:
        a, b = oracle.gen_inputs(n, n, n, phi, seed)
        rc, cf, plan, _ = oracle.emulate(a, b, n, n, n, passes=1, fixed_bits=54)
        rc2, ce, _, _ = oracle.emulate(a, b, n, n, n, passes=1, fixed_bits=54, exact=True)
        assert rc == 0 and rc2 == 0
        N = round_up(n, 64)
        _, dA, _ = oracle.scale(pad(a, n, n, N, N), N, N, 0, plan.shift)
        _, dB, _ = oracle.scale(pad(b, n, n, N, N), N, N, 1, plan.shift)
        KM = (plan.W_hi * 2.0 ** 32 + plan.W_lo) * 2.0 ** plan.qw
        g = 2 * plan.shift - (dA[:n, None] + dB[None, :n])
        bound = 2.0 ** -65 * KM * np.exp2(g.astype(np.float64)) + 2 * np.spacing(np.abs(cf.reshape(n, n)))
        assert np.all(np.abs(ce.reshape(n, n) - cf.reshape(n, n)) <= bound)
        # and the exact reconstruction is at least as accurate in the Frobenius norm
        hi, lo = oracle.dot2(a, b, n, n, n)
        assert oracle.accuracy(ce, hi, lo)[0] <= oracle.accuracy(cf, hi, lo)[0] * 1.0000001
