"""Scheme I INT8 on the host: the oracle against the reference's published device output, the
product's slice-count selection against the reference's own selection code compiled in place, and the
plan's feasibility errors (src/backend/ozaki1/plan.hpp:189-218)."""

import numpy as np
import pytest

from oracle_lib import pad, round_up

# tools/validated/quick.csv:12 — the reference device's Scheme I INT8 output for n=128, seed 7,
# uniform(-1,1), 8 slices.
PUBLISHED_I = {"n": 128, "seed": 7, "slices": 8, "output_hash": "6c9693442bfc11b0", "relative_fro": 4.68786522126e-17}


def test_oracle_reproduces_published_scheme_i_output(oracle):
    n = PUBLISHED_I["n"]
    a, b = oracle.gen_inputs(n, n, n, -1.0, PUBLISHED_I["seed"])
    c = oracle.i_emulate(a, b, n, n, n, PUBLISHED_I["slices"], exact=False)
    assert oracle.output_hash(c) == PUBLISHED_I["output_hash"]
    hi, lo = oracle.dot2(a, b, n, n, n)
    rel, _ = oracle.accuracy(c, hi, lo)
    assert rel == pytest.approx(PUBLISHED_I["relative_fro"], rel=1e-10)


def test_oracle_exact_recon_close_to_faithful(oracle):
    n = 128
    a, b = oracle.gen_inputs(n, n, n, 1.0, 3)
    faithful = oracle.i_emulate(a, b, n, n, n, 8, exact=False)
    exact = oracle.i_emulate(a, b, n, n, n, 8, exact=True)
    ulp = np.spacing(np.abs(exact))
    assert np.all(np.abs(faithful - exact) <= 2 * ulp)


def test_oracle_slices_are_digits_of_the_scaled_input(oracle):
    # sum_i d_i 254^-(i+1) reproduces x 2^delta to within 254^-p * 1/2 (balanced digits, clamp +-127).
    rng = np.random.default_rng(5)
    rows, cols, p = 4, 64, 6
    x = rng.standard_normal(rows * cols) * np.exp2(rng.integers(-20, 20, rows * cols))
    x = x.reshape(rows, cols)
    _, d, flags = oracle.scale(x.reshape(-1), rows, cols, 0, -1)
    assert flags == 0
    sl = oracle.i_slice(x.reshape(-1), rows, cols, 0, d, p).reshape(p, rows, cols).astype(np.float64)
    assert np.all(np.abs(sl) <= 127)
    approx = sum(sl[i] * 254.0 ** -(i + 1) for i in range(p))
    target = x * np.exp2(d.astype(np.float64))[:, None]
    assert np.all(np.abs(target) <= 0.5)
    assert np.all(np.abs(approx - target) <= 254.0 ** -p)


def _selection_cases(oracle):
    cases = []
    for phi in (-1.0, 0.5, 1.0, 2.0, 4.0):
        a, b = oracle.gen_inputs(128, 128, 128, phi, 7)
        cases.append((f"phi={phi}", a, b, 128, 128, 128))
    a, b = oracle.gen_inputs(100, 70, 45, -1.0, 11)
    cases.append(("ragged", a, b, 100, 70, 45))
    for mode in (2, 3, 4, 5):
        a, b = oracle.gen_pattern(65, 67, 97, mode)
        cases.append((f"pattern{mode}", a, b, 65, 67, 97))
    a, b = oracle.gen_pattern(33, 9, 300, 4)
    cases.append(("cancellation-long", a, b, 33, 9, 300))
    rng = np.random.default_rng(3)
    a = rng.standard_normal(70 * 200) * np.exp2(rng.integers(-60, 60, 70 * 200))
    b = rng.standard_normal(200 * 90)
    cases.append(("wide-range", a, b, 70, 90, 200))
    a = np.zeros(64 * 64)
    b = rng.standard_normal(64 * 64)
    cases.append(("zero-a", a, b, 64, 64, 64))
    a = np.full(3 * 5, 1.0 / 3.0)
    b = np.full(5 * 2, 3.0)
    cases.append(("constant", a, b, 3, 2, 5))
    return cases


def test_slice_selection_matches_reference(oracle, oztt, ref_plan1):
    for name, a, b, m, n, k in _selection_cases(oracle):
        M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
        want = ref_plan1.slices(pad(a, m, k, M, K), pad(b, k, n, K, N), M, N, K)
        plan = oztt.i_int8_plan(a, b, m, n, k)
        assert plan.p == want, name
        assert plan.auto_p == 1
        assert (plan.M, plan.N, plan.K) == (M, N, K)


def test_published_case_selection(oracle, oztt, ref_plan1):
    # The table run fixes 8 slices for INT8 (evaluation/evaluate.cpp:163); selected from the input, the
    # reference and the product both take 7 for this case.
    n = PUBLISHED_I["n"]
    a, b = oracle.gen_inputs(n, n, n, -1.0, PUBLISHED_I["seed"])
    assert oztt.i_int8_plan(a, b, n, n, n).p == ref_plan1.slices(a, b, n, n, n) == 7


def test_fixed_slices_are_kept(oztt):
    a, b = np.ones(8 * 8), np.ones(8 * 8)
    for p in (1, 2, 8, 13):
        plan = oztt.i_int8_plan(a, b, 8, 8, 8, slices=p)
        assert plan.p == p and plan.auto_p == 0


def test_k_blocking_is_rejected(oztt):
    # 8 slices: K_c <= 2^17 / 8 = 16384, so k = 16416 = 32 * 27 * 19 needs K blocks (the largest multiple
    # of 32 dividing it within the budget is 32 * 171 = 5472), which the INT8 path lacks.
    k = 16416
    a, b = np.ones(k), np.ones(k)
    with pytest.raises(RuntimeError, match="does not support K blocking, but k=16416 with 8 slices needs 3 K "
                                           "blocks of 5472 columns"):
        oztt.i_int8_plan(a, b, 1, 1, k, slices=8)
    # 16384 fits in one block.
    assert oztt.i_int8_plan(np.ones(16384), np.ones(16384), 1, 1, 16384, slices=8).p == 8


def test_horner_budget_is_rejected(oztt):
    # log2(32) + 15 log2(254) + 12 = 136.8 >= 128
    a, b = np.ones(32), np.ones(32)
    with pytest.raises(RuntimeError, match="reconstruction would overflow FP32 for k=32 with 15 slices"):
        oztt.i_int8_plan(a, b, 1, 1, 32, slices=15)
    assert oztt.i_int8_plan(a, b, 1, 1, 32, slices=13).p == 13


def test_plan_rejects_invalid_arguments(oztt):
    with pytest.raises(ValueError, match="at most 256"):
        oztt.i_int8_plan(np.ones(4), np.ones(4), 2, 2, 2, slices=257)


# ---- Scheme I with FP8 digits (radix 32, digits +-16, maxima truncated to BF16) -----------------------
FP8 = 4  # OZTT_FMT_FP8
# tools/validated/quick.csv:10 — the reference device's Scheme I FP8 output for n=128, seed 7, uniform(-1,1),
# 12 slices.
PUBLISHED_I_FP8 = {"n": 128, "seed": 7, "slices": 12, "output_hash": "4d24add106258287",
                   "relative_fro": 4.69453713108e-17}


def test_oracle_reproduces_published_scheme_i_fp8_output(oracle):
    n = PUBLISHED_I_FP8["n"]
    a, b = oracle.gen_inputs(n, n, n, -1.0, PUBLISHED_I_FP8["seed"])
    c = oracle.i_emulate(a, b, n, n, n, PUBLISHED_I_FP8["slices"], exact=False, fmt=FP8)
    assert oracle.output_hash(c) == PUBLISHED_I_FP8["output_hash"]
    hi, lo = oracle.dot2(a, b, n, n, n)
    rel, _ = oracle.accuracy(c, hi, lo)
    assert rel == pytest.approx(PUBLISHED_I_FP8["relative_fro"], rel=1e-10)


def test_oracle_fp8_slices_are_digits_of_the_scaled_input(oracle):
    # sum_i d_i 32^-(i+1) reproduces x 2^delta to within 32^-p * 16/31 (balanced digits, clamp +-16);
    # the truncated BF16 maxima leave |x 2^delta| up to (1 + 2^-7)/2, inside the span 16/31.
    rng = np.random.default_rng(6)
    rows, cols, p = 4, 64, 9
    x = rng.standard_normal(rows * cols) * np.exp2(rng.integers(-20, 20, rows * cols))
    x = x.reshape(rows, cols)
    _, d, flags = oracle.scale(x.reshape(-1), rows, cols, 0, -1, ceil=0)
    assert flags == 0
    sl = oracle.i_slice(x.reshape(-1), rows, cols, 0, d, p, fmt=FP8).reshape(p, rows, cols).astype(np.float64)
    assert np.all(np.abs(sl) <= 16)
    approx = sum(sl[i] * 32.0 ** -(i + 1) for i in range(p))
    target = x * np.exp2(d.astype(np.float64))[:, None]
    assert np.all(np.abs(target) <= 0.5 * (1 + 2.0 ** -7))
    assert np.all(np.abs(approx - target) <= 32.0 ** -p * 16 / 31 * (1 + 1e-12))


def test_oracle_fp8_exact_recon_close_to_faithful(oracle):
    n = 128
    a, b = oracle.gen_inputs(n, n, n, 1.0, 3)
    faithful = oracle.i_emulate(a, b, n, n, n, 12, exact=False, fmt=FP8)
    exact = oracle.i_emulate(a, b, n, n, n, 12, exact=True, fmt=FP8)
    assert np.all(np.abs(faithful - exact) <= 2 * np.spacing(np.abs(exact)))


def test_fp8_slice_selection_matches_reference(oracle, oztt, ref_plan1_f8):
    for name, a, b, m, n, k in _selection_cases(oracle):
        M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
        want = ref_plan1_f8.slices(pad(a, m, k, M, K), pad(b, k, n, K, N), M, N, K)
        plan = oztt.i_int8_plan(a, b, m, n, k, fmt=oztt.Format.FP8)
        assert plan.p == want, name
        assert (plan.format, plan.radix, plan.dmax) == (FP8, 32, 16)


def test_fp8_plan_feasibility(oztt):
    a, b = np.ones(32), np.ones(32)
    # log2(32) + 23 log2(32) + 12 = 132 >= 128: the Horner exponent budget
    with pytest.raises(RuntimeError, match=r"reconstruction would overflow FP32 for k=32 with 23 slices \(radix 32\)"):
        oztt.i_int8_plan(a, b, 1, 1, 32, slices=23, fmt=oztt.Format.FP8)
    assert oztt.i_int8_plan(a, b, 1, 1, 32, slices=22, fmt=oztt.Format.FP8).p == 22
    # K blocking is allowed for FP8 (no INT8-style rejection)
    k = 16416
    assert oztt.i_int8_plan(np.ones(k), np.ones(k), 1, 1, k, slices=8, fmt=oztt.Format.FP8).p == 8


# ---- Scheme I with BF16, FP16 and TF32 digits (radix 64, digits +-32) ---------------------------------
# tools/validated/quick.csv:2,4,6: the three formats share radix and digits, so their device outputs are
# identical: 10 slices, hash be6558fa9f435fa0, relative Frobenius error 4.69364573273e-17.
@pytest.mark.parametrize("fmt", [0, 1, 2])
def test_oracle_reproduces_published_radix64_output(oracle, fmt):
    n = 128
    a, b = oracle.gen_inputs(n, n, n, -1.0, 7)
    c = oracle.i_emulate(a, b, n, n, n, 10, exact=False, fmt=fmt)
    assert oracle.output_hash(c) == "be6558fa9f435fa0"
    hi, lo = oracle.dot2(a, b, n, n, n)
    assert oracle.accuracy(c, hi, lo)[0] == pytest.approx(4.69364573273e-17, rel=1e-10)


def test_radix64_slice_selection_matches_reference(oracle, oztt, ref_plan1_r64):
    for name, a, b, m, n, k in _selection_cases(oracle):
        M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
        want = ref_plan1_r64.slices(pad(a, m, k, M, K), pad(b, k, n, K, N), M, N, K)
        for fmt in (oztt.Format.BF16, oztt.Format.FP16, oztt.Format.TF32):
            plan = oztt.i_int8_plan(a, b, m, n, k, fmt=fmt)
            assert plan.p == want, (name, fmt)
            assert (plan.radix, plan.dmax) == (64, 32)
