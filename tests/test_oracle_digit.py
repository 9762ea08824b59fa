"""The oracle's Scheme II digit-format paths (FP8, BF16, FP16, TF32) pinned against the reference's
published device outputs.

CPU only. The digit plan comes from the library's digit planner (itself checked against the reference's
planner compiled for each format in test_planner_digit.py); the oracle then restates the digit split
(modslice_digit.cpp, sparse_fix.h), the digit products, the composition (compose.cpp; one-digit moduli
bypass it, RAWMASK) and the reconstruction from residues (recon_crt.cpp with IN_RESIDUE=1).
"""

import ctypes

import numpy as np
import pytest

import oztt_b200 as oztt
from oracle_lib import pad, round_up

# tools/validated/quick.csv:11 — II FP8, n=128, seed 7, uniform(-1,1), fixed_bits 54, one pass: 12 moduli,
# 36 digit products.
PUBLISHED_128 = {"output_hash": "20046e5bb3816cbb", "relative_fro": 4.6875329326e-17,
                 "effective_bits": 54.2439487868, "moduli": 12, "products": 36}
# tools/validated/quick.csv:3,5,7 — II BF16, FP16, TF32 with the same inputs and width (the route's default
# limit): (moduli, digit products, output hash, relative Frobenius error).
BF16, FP16, TF32 = 0, 1, 2
PUBLISHED_OTHER = {BF16: (12, 30, "13abe4ac7f292f42", 4.68753421163e-17),
                   FP16: (11, 31, "1811cf560959e61d", 4.68753617434e-17),
                   TF32: (11, 33, "9a8f2780d4b9976b", 4.6875327772e-17)}


def digit_case(oracle, m, n, k, phi, seed, **kw):
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    fp = oztt.digit_plan(a.reshape(m, k), b.reshape(k, n), m, n, k, **kw)
    return a, b, fp


def test_published_fp8_hash(oracle):
    n = 128
    a, b, fp = digit_case(oracle, n, n, n, -1.0, 7, reconstruction=1, fixed_bits=54)
    assert fp.base.S == PUBLISHED_128["moduli"] and fp.nprod == PUBLISHED_128["products"]
    assert fp.base.b == 54 and fp.base.two_pass == 0
    rc, c, err = oracle.digit_emulate(a, b, n, n, n, fp)
    assert rc == 0, err
    assert oracle.output_hash(c) == PUBLISHED_128["output_hash"]
    hi, lo = oracle.dot2(a, b, n, n, n)
    rel, ebits = oracle.accuracy(c, hi, lo)
    assert f"{rel:.10e}" == f"{PUBLISHED_128['relative_fro']:.10e}"
    assert abs(ebits - PUBLISHED_128["effective_bits"]) < 1e-9


@pytest.mark.parametrize("fmt", [BF16, FP16, TF32])
def test_published_digit_hashes(oracle, fmt):
    n = 128
    a, b, fp = digit_case(oracle, n, n, n, -1.0, 7, reconstruction=1, fixed_bits=54, fmt=fmt)
    S, nprod, h, rel = PUBLISHED_OTHER[fmt]
    assert (fp.base.S, fp.nprod, fp.base.b, fp.format) == (S, nprod, 54, fmt)
    if fmt != TF32:
        assert any(fp.mode[i] == oztt.SPLIT_ONE for i in range(fp.base.S))  # one-digit moduli in use
    rc, c, err = oracle.digit_emulate(a, b, n, n, n, fp)
    assert rc == 0, err
    assert oracle.output_hash(c) == h
    hi, lo = oracle.dot2(a, b, n, n, n)
    assert f"{oracle.accuracy(c, hi, lo)[0]:.10e}" == f"{rel:.10e}"


def test_plan_uses_every_splitting_method(oracle):
    """The published plan mixes sparse squares (SQS), squares (SQ) and Karatsuba (KAR); the digit planes of
    every element are integers that e4m3 represents exactly."""
    n = 128
    a, b, fp = digit_case(oracle, n, n, n, -1.0, 7, reconstruction=1, fixed_bits=54)
    modes = {fp.mode[i] for i in range(fp.base.S)}
    assert {oztt.SPLIT_SQ, oztt.SPLIT_KAR, oztt.SPLIT_SQS} <= modes
    crt = oracle.crt_plan([fp.base.moduli[i] for i in range(fp.base.S)], fp.base.b, fp.base.two_pass)
    _, dA, _ = oracle.scale(a, n, n, 0, crt.shift)
    bad, planes = oracle.digit_split(a, n, n, 0, dA, crt, fp)
    assert bad == 0
    vals = np.unique(planes)
    assert np.all((np.abs(vals) <= 16) | ((np.abs(vals) <= 32) & (vals % 2 == 0)))
    assert np.abs(vals).max() > 16  # the sparse digits are in use


@pytest.mark.parametrize("m,n,k,phi,seed,passes", [(96, 160, 200, 0.5, 3, 1), (64, 64, 1000, 2.0, 5, 2),
                                                   (130, 70, 64, -1.0, 11, 0)])
def test_faithful_and_exact_agree(oracle, m, n, k, phi, seed, passes):
    """The reference's triple-float reconstruction and the exact one agree within the faithful pass's error:
    2^-65 (one pass) or 2^-90 (two passes) times M 2^-2b 2^(2 shift - dA_i - dB_j), plus 2 ulp."""
    a, b, fp = digit_case(oracle, m, n, k, phi, seed, reconstruction=passes)
    rc, cf, err = oracle.digit_emulate(a, b, m, n, k, fp)
    assert rc == 0, err
    rc, ce, err = oracle.digit_emulate(a, b, m, n, k, fp, exact=True)
    assert rc == 0, err
    hi, lo = oracle.dot2(a, b, m, n, k)
    crt = oracle.crt_plan([fp.base.moduli[i] for i in range(fp.base.S)], fp.base.b, fp.base.two_pass)
    M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
    _, dA, _ = oracle.scale(pad(a, m, k, M, K), M, K, 0, crt.shift)
    _, dB, _ = oracle.scale(pad(b, k, n, K, N), K, N, 1, crt.shift)
    KM = (crt.W_hi * 2.0 ** 32 + crt.W_lo) * 2.0 ** crt.qw
    g = 2 * crt.shift - (dA[:m, None] + dB[None, :n])
    tol = (2.0 ** -90 if crt.two_pass else 2.0 ** -65) * KM * np.exp2(g.astype(np.float64))
    assert np.all(np.abs(cf - ce).reshape(m, n) <= tol + 2 * np.spacing(np.abs(cf.reshape(m, n))))
    rel, _ = oracle.accuracy(ce, hi, lo)
    assert rel < 1e-15


def test_compose_split_matches_fold_first(oracle):
    """Both composition methods (reduce first, or split at 2^12 with coeff_hi) give the same residue class:
    with the exact reconstruction the outputs are identical."""
    m = n = 64
    k = 256
    a, b, fp = digit_case(oracle, m, n, k, 1.0, 9)
    rc, c1, err = oracle.digit_emulate(a, b, m, n, k, fp, exact=True)
    assert rc == 0, err
    fp2 = oztt.DigitPlan()
    ctypes.memmove(ctypes.byref(fp2), ctypes.byref(fp), ctypes.sizeof(fp))
    fp2.fold_first = 1 - fp.fold_first
    rc, c2, err = oracle.digit_emulate(a, b, m, n, k, fp2, exact=True)
    assert rc == 0, err
    assert np.array_equal(c1.view(np.uint64), c2.view(np.uint64))


@pytest.mark.parametrize("fmt", [4, BF16, FP16, TF32])
def test_reference_plan_reproduces_hash(oracle, ref_plan_digit, fmt):
    """With the reference's own planner (compiled in place for the format) the oracle reproduces the hash."""
    n = 128
    a, b = oracle.gen_inputs(n, n, n, -1.0, 7)
    rc, fp = ref_plan_digit(fmt).plan(pad(a, n, n, n, n), pad(b, n, n, n, n), n, n, n, oztt.DigitPlan, 0, 1, 54)
    assert rc == 0
    rc, c, err = oracle.digit_emulate(a, b, n, n, n, fp)
    assert rc == 0, err
    assert oracle.output_hash(c) == (PUBLISHED_128["output_hash"] if fmt == 4 else PUBLISHED_OTHER[fmt][2])
