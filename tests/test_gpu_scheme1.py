"""Scheme I (INT8 and FP8 slices) on the B200, stage by stage and end to end, against the oracle.

Every call goes through the C ABI of liboztt.so. Bars:
  * slices (radix-254 digits of every element for INT8, radix-32 digits for FP8): bit-exact against the
    oracle's restatement of the reference slicer (slice_tf_body.h with tfMulR / tfMulP2);
  * diagonal products P_d (int32): bit-exact;
  * the FP64 output: bit-exact against the oracle's restatement of the B200 exact Horner
    reconstruction, and within |C - C_ref| <= 2 ulp(C) + 2^-58 (|A| |B|)_ij of the reference's own
    triple-float reconstruction;
  * the acceptance cases of the reference's tests/correctness.cpp (relative Frobenius error <= 8 eps).
"""

import numpy as np
import pytest
import torch

from oracle_lib import pad, round_up

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def stream():
    return torch.cuda.current_stream().cuda_stream


INT8, FP8, BF16 = 5, 4, 0  # OZTT_FMT_* values (BF16 stands for the radix-64 formats BF16, FP16, TF32)
FORMATS = [INT8, FP8, BF16]
CEIL = {INT8: 1, FP8: 0, BF16: 0}  # BF16 rounding of the maxima: up for INT8, truncated for the FP formats


def gpu_deltas(oztt, x, rows, cols, col_mode, fmt=INT8):
    X = dev(x)
    nout = cols if col_mode else rows
    delta = torch.zeros(nout, dtype=torch.int32, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    name = "oztt_i_scale_cols" if col_mode else "oztt_i_scale_rows"
    oztt.call(name, X.data_ptr(), rows, cols, cols, fmt, delta.data_ptr(), flags.data_ptr(), stream())
    return X, delta, flags


def hard_matrix(rng, rows, cols):
    """Random values plus the slicer's corner cases: exact powers of two (a digit of exactly 127 after
    the first step), values just around the row maximum, halves of 254^-i (rounding ties of later
    digits), tiny elements beside large ones (underflow of the triple-float limbs), zeros, negatives."""
    x = rng.standard_normal(rows * cols) * np.exp2(rng.integers(-30, 30, rows * cols))
    x = x.reshape(rows, cols)
    x[:, 0] = np.exp2(rng.integers(-5, 5, rows)).astype(np.float64)
    if cols > 3:
        x[:, 1] = x[:, 0] * (1 - 2.0 ** -52)
        x[:, 2] = -x[:, 0] * (0.5 + 0.5 / 254)
        x[:, 3] = x[:, 0] * 2.0 ** -200
    if cols > 8:
        x[:, 4] = 0.0
        x[:, 5] = x[:, 0] * (0.5 / 254 + 0.5 / 254 ** 2)
        x[:, 6] = x[:, 0] * (1.0 / 254 ** 3) * 0.5
        x[:, 7] = 5e-324
        x[:, 8] = -x[:, 0] * 2.0 ** -60
    if rows > 2:
        x[1, :] = 0.0
    return x.reshape(-1)


SLICE_CASES = [(64, 64, 8), (33, 100, 7), (257, 129, 13), (5, 4097, 3), (128, 256, 1), (300, 45, 16)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,k,p", SLICE_CASES)
def test_slice_rows_match_oracle(oztt, oracle, cuda, m, k, p, fmt):
    rng = np.random.default_rng(m * 1000 + k)
    a = hard_matrix(rng, m, k)
    A, delta, flags = gpu_deltas(oztt, a, m, k, 0, fmt)
    _, od, ofl = oracle.scale(a, m, k, 0, -1, ceil=CEIL[fmt])
    mp, kp = round_up(m, 128), round_up(k, 128)
    planes = torch.full((p * mp * kp,), 99, dtype=torch.int8, device="cuda")
    oztt.call("oztt_i_slice_rows", A.data_ptr(), m, k, k, delta.data_ptr(), p, fmt, planes.data_ptr(), mp, kp,
              stream())
    torch.cuda.synchronize()
    assert np.array_equal(delta.cpu().numpy(), od) and int(flags.cpu()[0]) == ofl
    got = planes.cpu().numpy().reshape(p, mp, kp)
    want = oracle.i_slice(a, m, k, 0, od, p, fmt=fmt).reshape(p, m, k)
    assert np.array_equal(got[:, :m, :k], want)
    assert not got[:, m:, :].any() and not got[:, :, k:].any()


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("k,n,p", SLICE_CASES)
def test_slice_cols_match_oracle(oztt, oracle, cuda, k, n, p, fmt):
    rng = np.random.default_rng(k * 1000 + n + 1)
    b = np.ascontiguousarray(hard_matrix(rng, n, k).reshape(n, k).T).reshape(-1)
    B, delta, flags = gpu_deltas(oztt, b, k, n, 1, fmt)
    _, od, ofl = oracle.scale(b, k, n, 1, -1, ceil=CEIL[fmt])
    np_, kp = round_up(n, 256), round_up(k, 128)
    planes = torch.full((p * np_ * kp,), 99, dtype=torch.int8, device="cuda")
    oztt.call("oztt_i_slice_cols", B.data_ptr(), k, n, n, delta.data_ptr(), p, fmt, planes.data_ptr(), np_, kp,
              stream())
    torch.cuda.synchronize()
    assert np.array_equal(delta.cpu().numpy(), od) and int(flags.cpu()[0]) == ofl
    got = planes.cpu().numpy().reshape(p, np_, kp)
    want = oracle.i_slice(b, k, n, 1, od, p, fmt=fmt).reshape(p, n, k)
    assert np.array_equal(got[:, :n, :k], want)
    assert not got[:, n:, :].any() and not got[:, :, k:].any()


def gpu_diag(oztt, sa, sb, mp, np_, kp, p):
    SA, SB = dev(sa), dev(sb)
    out = torch.full((p * mp * np_,), 7, dtype=torch.int32, device="cuda")
    oztt.call("oztt_i_diag_gemm", SA.data_ptr(), SB.data_ptr(), mp, np_, kp, p, out.data_ptr(), stream())
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("mp,np_,kp,p", [(128, 256, 128, 1), (128, 256, 256, 4), (384, 512, 640, 8),
                                         (256, 768, 128, 13), (1280, 256, 384, 3)])
def test_diag_gemm_matches_oracle(oztt, oracle, cuda, mp, np_, kp, p):
    rng = np.random.default_rng(mp + np_ + kp + p)
    sa = rng.integers(-127, 128, p * mp * kp, dtype=np.int8)
    sb = rng.integers(-127, 128, p * np_ * kp, dtype=np.int8)
    assert np.array_equal(gpu_diag(oztt, sa, sb, mp, np_, kp, p), oracle.i_gemm(sa, sb, p, mp, np_, kp))


def test_diag_gemm_at_the_int32_budget(oztt, cuda):
    # 8 slices, K = 2^17 / 8: every product is +127 * +127 (or -127 * +127), the largest diagonal sum is
    # 8 * 16384 * 127^2 = 2113667072 < 2^31 - 1.
    mp, np_, kp, p = 128, 256, 16384, 8
    sa = np.full(p * mp * kp, 127, dtype=np.int8)
    sa.reshape(p, mp, kp)[:, 1::2, :] = -127
    sb = np.full(p * np_ * kp, 127, dtype=np.int8)
    got = gpu_diag(oztt, sa, sb, mp, np_, kp, p).reshape(p, mp, np_)
    for d in range(p):
        want = (d + 1) * kp * 127 * 127
        assert np.all(got[d, 0::2, :] == want) and np.all(got[d, 1::2, :] == -want)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,n,p", [(64, 64, 1), (100, 70, 5), (128, 256, 8), (33, 300, 13)])
def test_recon_matches_oracle(oztt, oracle, cuda, m, n, p, fmt):
    rng = np.random.default_rng(m * n + p)
    mp, np_ = round_up(m, 128), round_up(n, 256)
    K = 2048
    radix, dmax = {INT8: (254, 127), FP8: (32, 16), BF16: (64, 32)}[fmt]
    bound = np.array([(d + 1) * K * dmax * dmax for d in range(p)], dtype=np.int64)
    pd = (rng.uniform(-1, 1, (p, mp, np_)) * bound[:, None, None] * rng.uniform(0, 1, (p, 1, 1))).astype(np.int32)
    pd[:, 0, 0] = 0                     # zero result
    pd[:, 0, 1] = bound.astype(np.int32)  # largest positive
    pd[:, 0, 2] = -bound.astype(np.int32)
    pd[0, 0, 3], pd[1:, 0, 3] = 1, 0    # one unit in the top diagonal only
    dA = rng.integers(-40, 40, mp).astype(np.int32)
    dB = rng.integers(-40, 40, np_).astype(np.int32)
    dA[2] = 1000                        # results far below 2^-1022: flushed to zero
    PD, DA, DB = dev(pd.reshape(-1)), dev(dA), dev(dB)
    c = torch.full((m * n,), 3.0, dtype=torch.float64, device="cuda")
    oztt.call("oztt_i_recon", PD.data_ptr(), mp, np_, DA.data_ptr(), DB.data_ptr(), p, fmt, c.data_ptr(), m, n, n,
              stream())
    torch.cuda.synchronize()
    got = c.cpu().numpy().reshape(m, n)
    exact = oracle.i_recon(pd.reshape(-1), p, mp, np_, dA, dB, exact=True, fmt=fmt).reshape(mp, np_)[:m, :n]
    assert np.array_equal(got.view(np.uint64), exact.view(np.uint64))
    faithful = oracle.i_recon(pd.reshape(-1), p, mp, np_, dA, dB, exact=False, fmt=fmt, K=K).reshape(mp, np_)[:m, :n]
    # magnitude bound of the sum: sum_d |P_d| r^(L-d) r^-(L+2) 2^-(dA+dB)
    w = np.array([float(radix) ** (-(d + 2)) for d in range(p)])
    mag = np.tensordot(w, np.abs(pd[:, :m, :n].astype(np.float64)), axes=1)
    mag *= np.exp2(-(dA[:m, None] + dB[None, :n]).astype(np.float64))
    assert np.all(np.abs(got - faithful) <= 2 * np.spacing(np.abs(got)) + 2.0 ** -58 * mag)


def run_gpu(oztt, a, b, m, n, k, p=0, fmt=INT8):
    plan = oztt.i_int8_plan(a, b, m, n, k, slices=p, fmt=fmt)
    return oztt.i_int8_run(a, b, m, n, k, plan), plan


def absprod(a, b, m, n, k):
    return np.abs(a.reshape(m, k)) @ np.abs(b.reshape(k, n))


PIPE_CASES = [("uniform", 128, 128, 128, -1.0, 8), ("phi1", 100, 70, 45, 1.0, 0), ("phi4", 64, 200, 300, 4.0, 0),
              ("tall", 1000, 3, 64, 0.5, 6), ("wide", 3, 1000, 96, -1.0, 0), ("one", 1, 1, 1, -1.0, 2)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("name,m,n,k,phi,p", PIPE_CASES)
def test_pipeline_matches_oracle(oztt, oracle, cuda, name, m, n, k, phi, p, fmt):
    a, b = oracle.gen_inputs(m, n, k, phi, 17)
    p = p if fmt == INT8 or p == 0 else p + {FP8: 4, BF16: 2}[fmt]  # radix 32/64 carry 5/6 bits a slice, 254 ~8
    c, plan = run_gpu(oztt, a, b, m, n, k, p, fmt)
    assert p == 0 or plan.p == p
    exact = oracle.i_emulate(a, b, m, n, k, plan.p, exact=True, fmt=fmt)
    assert np.array_equal(c.view(np.uint64), exact.view(np.uint64)), name
    faithful = oracle.i_emulate(a, b, m, n, k, plan.p, exact=False, fmt=fmt)
    tol = 2 * np.spacing(np.abs(c)) + 2.0 ** -58 * absprod(a, b, m, n, k).reshape(-1)
    assert np.all(np.abs(c - faithful) <= tol), name


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("mode", [2, 3, 4, 5, 6, 7])
def test_pipeline_patterns(oztt, oracle, cuda, mode, fmt):
    m, n, k = (65, 67, 97) if mode < 6 else (1, 1, 1)
    a, b = oracle.gen_pattern(m, n, k, mode)
    c, plan = run_gpu(oztt, a, b, m, n, k, fmt=fmt)
    exact = oracle.i_emulate(a, b, m, n, k, plan.p, exact=True, fmt=fmt)
    assert np.array_equal(c.view(np.uint64), exact.view(np.uint64))


def test_published_case(oztt, oracle, cuda):
    # tools/validated/quick.csv:12: n=128, seed 7, 8 slices; the reference's device output has relative
    # Frobenius error 4.68786522126e-17 against Dot2 and hash 6c9693442bfc11b0.
    n = 128
    a, b = oracle.gen_inputs(n, n, n, -1.0, 7)
    c, _ = run_gpu(oztt, a, b, n, n, n, 8)
    ref = oracle.i_emulate(a, b, n, n, n, 8, exact=False)
    assert oracle.output_hash(ref) == "6c9693442bfc11b0"
    assert np.all(np.abs(c - ref) <= 2 * np.spacing(np.abs(c)))
    hi, lo = oracle.dot2(a, b, n, n, n)
    rel, _ = oracle.accuracy(c, hi, lo)
    assert abs(rel - 4.68786522126e-17) <= 1e-3 * 4.68786522126e-17


def test_device_entry_matches_host_entry(oztt, oracle, cuda):
    m, n, k = 200, 300, 160
    a, b = oracle.gen_inputs(m, n, k, 0.5, 9)
    host, plan = run_gpu(oztt, a, b, m, n, k)
    A, B = dev(a), dev(b)
    C = torch.zeros(m * n, dtype=torch.float64, device="cuda")
    ms = oztt.i_int8_run_device(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, plan, stream(), timed=True)
    assert len(ms) == 5 and all(t >= 0 for t in ms)
    assert np.array_equal(C.cpu().numpy().view(np.uint64), host.view(np.uint64))


def test_context_scheme_i(oztt, oracle, cuda):
    ctx = oztt.Context()
    m, n, k = 65, 67, 97
    a, b = oracle.gen_inputs(m, n, k, 1.0, 4)
    opts = oztt.Options(scheme=oztt.Scheme.I, format=oztt.Format.INT8)
    c = np.empty(m * n)
    info = ctx.gemm(a, b, c, m, n, k, opts)
    plan = oztt.i_int8_plan(a, b, m, n, k)
    assert info.scheme == oztt.Scheme.I and info.slices == plan.p and info.moduli == 0
    assert (info.padded_m, info.padded_n, info.padded_k) == (128, 128, 128)
    exact = oracle.i_emulate(a, b, m, n, k, plan.p, exact=True)
    assert np.array_equal(c.view(np.uint64), exact.view(np.uint64))
    hi, lo = oracle.dot2(a, b, m, n, k)
    assert oracle.accuracy(c, hi, lo)[0] <= 8 * np.finfo(np.float64).eps
    with pytest.raises(RuntimeError, match="reconstruction would overflow FP32"):
        ctx.multiply(a, b, m, n, k, oztt.Options(scheme=oztt.Scheme.I, format=oztt.Format.INT8, slices=15))


def test_published_case_fp8(oztt, oracle, cuda):
    # tools/validated/quick.csv:10: Scheme I FP8, n=128, seed 7, 12 slices; relative Frobenius error
    # 4.69453713108e-17 against Dot2 and hash 4d24add106258287 on the reference device.
    n = 128
    a, b = oracle.gen_inputs(n, n, n, -1.0, 7)
    c, _ = run_gpu(oztt, a, b, n, n, n, 12, FP8)
    ref = oracle.i_emulate(a, b, n, n, n, 12, exact=False, fmt=FP8)
    assert oracle.output_hash(ref) == "4d24add106258287"
    assert np.all(np.abs(c - ref) <= 2 * np.spacing(np.abs(c)))
    hi, lo = oracle.dot2(a, b, n, n, n)
    rel, _ = oracle.accuracy(c, hi, lo)
    assert abs(rel - 4.69453713108e-17) <= 1e-3 * 4.69453713108e-17


def test_context_scheme_i_fp8(oztt, oracle, cuda):
    ctx = oztt.Context()
    m, n, k = 65, 67, 97
    a, b = oracle.gen_inputs(m, n, k, 1.0, 4)
    c = np.empty(m * n)
    info = ctx.gemm(a, b, c, m, n, k, oztt.Options(scheme=oztt.Scheme.I, format=oztt.Format.FP8))
    plan = oztt.i_int8_plan(a, b, m, n, k, fmt=oztt.Format.FP8)
    assert info.scheme == oztt.Scheme.I and info.format == oztt.Format.FP8 and info.slices == plan.p
    exact = oracle.i_emulate(a, b, m, n, k, plan.p, exact=True, fmt=FP8)
    assert np.array_equal(c.view(np.uint64), exact.view(np.uint64))
    hi, lo = oracle.dot2(a, b, m, n, k)
    assert oracle.accuracy(c, hi, lo)[0] <= 8 * np.finfo(np.float64).eps
    # the fixed slice count of the reference's test for FP8 (tests/correctness.cpp:280)
    c12 = ctx.multiply(a, b, m, n, k, oztt.Options(scheme=oztt.Scheme.I, format=oztt.Format.FP8, slices=12))
    assert np.array_equal(c12.view(np.uint64), oracle.i_emulate(a, b, m, n, k, 12, exact=True, fmt=FP8).view(np.uint64))


# ---- slice selection with the per-element statistics measured on the device (plan1_dev.cu) --------------
SELECT_CASES = [(5, 150, 90, 260, 0.5, 41, None), (5, 129, 65, 200, 4.0, 42, "tiny"), (4, 97, 131, 77, 1.0, 43, None),
                (0, 200, 72, 256, 2.0, 44, "zeros"), (5, 300, 280, 1000, 8.0, 45, None), (2, 64, 64, 64, -1.0, 46, None),
                (4, 1, 70, 1000, 1.0, 47, "zeros"), (0, 513, 257, 129, 0.5, 48, "tiny")]


@pytest.mark.parametrize("fmt,m,n,k,phi,seed,extra", SELECT_CASES)
def test_device_selection_equals_host(oztt, oracle, cuda, fmt, m, n, k, phi, seed, extra):
    """Model (1)'s error vector and the ||C||_F^2 estimate measured on the device equal the host planner's to
    the bit, and so does the plan (zero rows and columns, elements below 2^-383 that send the device
    statistics to their scale-first recomputation, every radix)."""
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    if extra == "zeros":
        a[: k] = 0.0
        b[::5] = 0.0
    if extra == "tiny":
        a[3], b[7] = 2.0 ** -500, -(2.0 ** -450)
    A, B = dev(a), dev(b)
    host = oztt.i_model1_errors(a, b, m, n, k, fmt=fmt)
    devv = oztt.i_model1_errors(None, None, m, n, k, fmt=fmt, a_dev=A.data_ptr(), b_dev=B.data_ptr(),
                                stream=stream())
    assert np.array_equal(host.view(np.uint64), devv.view(np.uint64))
    hp = oztt.i_int8_plan(a, b, m, n, k, fmt=fmt)
    dp = oztt.i_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, fmt=fmt, stream=stream())
    assert bytes(hp) == bytes(dp)


@pytest.mark.parametrize("fmt", [5, 4, 0])
def test_context_scheme_i_device_selection(oztt, oracle, cuda, fmt):
    """Context::gemm's Scheme I call selects the slice count on the device and runs on the resident operands:
    the host plan's p and the bits of the host-planned run."""
    m, n, k = 333, 222, 444
    a, b = oracle.gen_inputs(m, n, k, 1.0, 49)
    plan = oztt.i_int8_plan(a, b, m, n, k, fmt=fmt)
    c = np.empty(m * n)
    info = oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(scheme=oztt.Scheme.I, format=fmt))
    assert info.slices == plan.p
    ref = oztt.i_int8_run(a, b, m, n, k, plan)
    assert np.array_equal(c.view(np.uint64), ref.view(np.uint64))


@pytest.mark.parametrize("fmt", [5, 0])
def test_context_scheme_i_streamed_bands(oztt, oracle, cuda, fmt):
    """Context::gemm's streamed Scheme I call over several column blocks of both operands and two row bands
    (the last ragged): the host plan's p and the bits of the host-planned run; value errors come from the
    measured maxima in the reference's order, before a fixed-slice feasibility error."""
    m, n, k = 4500, 2048, 4608
    a, b = oracle.gen_inputs(m, n, k, 0.5, 51)
    plan = oztt.i_int8_plan(a, b, m, n, k, fmt=fmt)
    c = np.full(m * n, 123.0)
    ctx = oztt.Context()
    info = ctx.gemm(a, b, c, m, n, k, oztt.Options(scheme=oztt.Scheme.I, format=fmt))
    assert info.slices == plan.p
    ref = oztt.i_int8_run(a, b, m, n, k, plan)
    assert np.array_equal(c.view(np.uint64), ref.view(np.uint64))
    assert oztt.ii_int8_last_phases()["bands"] == 2
    a[17] = np.nan
    c2 = np.full(64 * 64, 123.0)
    small_a, small_b = a[: 64 * 64].copy(), b[: 64 * 64].copy()
    with pytest.raises(ValueError, match="A contains NaN or infinity"):
        ctx.gemm(small_a, small_b, c2, 64, 64, 64, oztt.Options(scheme=oztt.Scheme.I, format=fmt))
    with pytest.raises(ValueError, match="A contains NaN or infinity"):  # before the infeasible 255 slices
        ctx.gemm(small_a, small_b, c2, 64, 64, 64, oztt.Options(scheme=oztt.Scheme.I, format=fmt, slices=255))
    assert np.all(c2 == 123.0)
