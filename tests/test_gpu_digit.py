"""Scheme II with the digit formats (FP8 e4m3, BF16, FP16, TF32) on the B200, stage by stage and end to end,
against the oracle.

Every call goes through the C ABI of liboztt.so. Bars:
  * digit planes (every splitting method: ONE, SQ, KAR, WIDE, SQS) and the GEMM outputs P_o (int32):
    bit-exact against the oracle's restatement of modslice_digit.cpp / sparse_fix.h and of the digit products;
  * the CRT digits of the fused composition: equal to (sum_o coeff_o P_o) y_s mod m_s computed on the host
    from the oracle's P_o, and in the same residue class as the oracle's restatement of compose.cpp;
  * the FP64 output: bit-exact against the oracle's exact CRT from residues, and within the faithful
    tolerance of the reference's own (triple-float) reconstruction;
  * the published device hashes at n=128 (tools/validated/quick.csv:3,5,7,11) through the GPU digit planes
    and products with the reference's composition and reconstruction restated on the host, and the
    acceptance cases of the reference's tests/correctness.cpp through the public API for every format.
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


FP8, BF16, FP16, TF32 = 4, 0, 1, 2  # OZTT_FMT_* values
FORMATS = [FP8, BF16, FP16, TF32]


def plan_and_crt(oztt, oracle, a, b, m, n, k, **kw):
    fp = oztt.digit_plan(a.reshape(m, k), b.reshape(k, n), m, n, k, **kw)
    crt = oracle.crt_plan([fp.base.moduli[i] for i in range(fp.base.S)], fp.base.b, fp.base.two_pass)
    return fp, crt


def gpu_scale(oztt, X, rows, cols, col_mode, shift):
    nout = cols if col_mode else rows
    delta = torch.zeros(nout, dtype=torch.int32, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    name = "oztt_ii_scale_cols" if col_mode else "oztt_ii_scale_rows"
    oztt.call(name, X.data_ptr(), rows, cols, cols, shift, delta.data_ptr(), None, flags.data_ptr(), stream())
    return delta


def gpu_digits(oztt, X, rows, cols, col_mode, delta, fp):
    """Digit planes of A (rows x cols) or of B (rows = k, cols = n) as the GEMM reads them."""
    if col_mode:
        npad, kpad = round_up(cols, 256), round_up(rows, 128)
        out = torch.full((fp.nplane * npad * kpad,), 77, dtype=torch.int8, device="cuda")
        oztt.call("oztt_ii_digit_split_cols", X.data_ptr(), rows, cols, cols, delta.data_ptr(), fp, out.data_ptr(), npad,
                  kpad, stream())
        return out, npad, kpad
    mpad, kpad = round_up(rows, 128), round_up(cols, 128)
    out = torch.full((fp.nplane * mpad * kpad,), 77, dtype=torch.int8, device="cuda")
    oztt.call("oztt_ii_digit_split_rows", X.data_ptr(), rows, cols, cols, delta.data_ptr(), fp, out.data_ptr(), mpad, kpad,
              stream())
    return out, mpad, kpad


def faithful_bound(oracle, a, b, m, n, k, crt, cf):
    """|C - C_reference| allowed against the reference's triple-float reconstruction: 2^-65 (one pass) or
    2^-90 (two passes) times M 2^-2b 2^(2 shift - dA_i - dB_j), plus 2 ulp of C_reference."""
    M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
    _, dA, _ = oracle.scale(pad(a, m, k, M, K), M, K, 0, crt.shift)
    _, dB, _ = oracle.scale(pad(b, k, n, K, N), K, N, 1, crt.shift)
    KM = (crt.W_hi * 2.0 ** 32 + crt.W_lo) * 2.0 ** crt.qw
    g = 2 * crt.shift - (dA[:m, None] + dB[None, :n])
    tol = (2.0 ** -90 if crt.two_pass else 2.0 ** -65) * KM * np.exp2(g.astype(np.float64))
    return tol + 2 * np.spacing(np.abs(cf.reshape(m, n)))


def modes_of(fp):
    return {fp.mode[i] for i in range(fp.base.S)}


# (m, n, k, phi, seed, plan arguments): the published plan (SQS, SQ, KAR), a WIDE modulus (K=1024, b=64, 16
# moduli), all four methods (b=99, 24 moduli, nd=5), dense digits at K=16384 (SQ, KAR), ragged shapes.
SPLIT_CASES = [
    (128, 128, 128, -1.0, 7, dict(reconstruction=1, fixed_bits=54)),
    (96, 80, 1024, 0.5, 3, dict(reconstruction=1, fixed_bits=64, max_moduli=16)),
    (70, 90, 1024, 4.0, 4, dict(reconstruction=1, fixed_bits=99, max_moduli=24)),
    (64, 64, 16384, 1.0, 5, dict(reconstruction=1, fixed_bits=54)),
    (257, 33, 300, 2.0, 6, dict()),
]


@pytest.mark.parametrize("fmt", [FP8, BF16, TF32])
@pytest.mark.parametrize("m,n,k,phi,seed,kw", SPLIT_CASES)
def test_digit_split_matches_oracle(oztt, oracle, cuda, m, n, k, phi, seed, kw, fmt):
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    if fmt != FP8 and k >= 16384:
        k = 8192  # the 32-digit routes need K * 32^2 <= 2^24
    fp, crt = plan_and_crt(oztt, oracle, a[:m * k], b[:k * n], m, n, k, fmt=fmt, **kw)
    a, b = a[:m * k], b[:k * n]
    A, B = dev(a), dev(b)
    dA = gpu_scale(oztt, A, m, k, 0, fp.base.shift)
    dB = gpu_scale(oztt, B, k, n, 1, fp.base.shift)
    _, oda, _ = oracle.scale(a, m, k, 0, crt.shift)
    _, odb, _ = oracle.scale(b, k, n, 1, crt.shift)
    assert np.array_equal(dA.cpu().numpy(), oda) and np.array_equal(dB.cpu().numpy(), odb)
    ga, mp, kp = gpu_digits(oztt, A, m, k, 0, dA, fp)
    gb, np_, kp2 = gpu_digits(oztt, B, k, n, 1, dB, fp)
    torch.cuda.synchronize()
    bad, ra = oracle.digit_split(a, m, k, 0, oda, crt, fp)
    assert bad == 0
    bad, rb = oracle.digit_split(b, k, n, 1, odb, crt, fp)
    assert bad == 0
    ga = ga.view(fp.nplane, mp, kp).cpu().numpy()
    gb = gb.view(fp.nplane, np_, kp2).cpu().numpy()
    assert np.array_equal(ga[:, :m, :k], ra.reshape(fp.nplane, m, k))
    assert np.array_equal(gb[:, :n, :k], rb.reshape(fp.nplane, n, k))
    # padding is written as zero digits
    assert not ga[:, m:, :].any() and not ga[:, :, k:].any()
    assert not gb[:, n:, :].any() and not gb[:, :, k:].any()


def test_split_cases_cover_every_method(oztt, oracle):
    seen = set()
    for fmt in (FP8, BF16):
        for m, n, k, phi, seed, kw in SPLIT_CASES:
            if fmt != FP8 and k >= 16384:
                k = 8192
            fp = oztt.digit_plan(None, None, m, n, k, fmt=fmt, **kw) if kw.get("fixed_bits") else None
            if fp is not None:
                seen |= modes_of(fp)
    assert seen == {oztt.SPLIT_SQ, oztt.SPLIT_KAR, oztt.SPLIT_WIDE, oztt.SPLIT_SQS, oztt.SPLIT_ONE}


def digit_case(oztt, oracle, m, n, k, phi, seed, kw, fmt=FP8):
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    fp, crt = plan_and_crt(oztt, oracle, a, b, m, n, k, fmt=fmt, **kw)
    A, B = dev(a), dev(b)
    dA = gpu_scale(oztt, A, m, k, 0, fp.base.shift)
    dB = gpu_scale(oztt, B, k, n, 1, fp.base.shift)
    ga, mp, kp = gpu_digits(oztt, A, m, k, 0, dA, fp)
    gb, np_, _ = gpu_digits(oztt, B, k, n, 1, dB, fp)
    return a, b, fp, crt, dA, dB, ga, gb, mp, np_, kp


GEMM_CASES = [(128, 256, 128, -1.0, 7, dict(reconstruction=1, fixed_bits=54)),
              (128, 256, 1024, 0.5, 3, dict(reconstruction=1, fixed_bits=64, max_moduli=16)),
              (130, 260, 500, 4.0, 4, dict(reconstruction=1, fixed_bits=99, max_moduli=24)),
              (128, 256, 2048, 1.0, 8, dict())]


@pytest.mark.parametrize("fmt", [FP8, BF16, TF32])
@pytest.mark.parametrize("m,n,k,phi,seed,kw", GEMM_CASES)
def test_digit_gemm_matches_oracle(oztt, oracle, cuda, m, n, k, phi, seed, kw, fmt):
    a, b, fp, crt, dA, dB, ga, gb, mp, np_, kp = digit_case(oztt, oracle, m, n, k, phi, seed, kw, fmt)
    P = torch.empty(fp.nout * mp * np_, dtype=torch.int32, device="cuda")
    oztt.call("oztt_ii_digit_gemm", ga.data_ptr(), gb.data_ptr(), mp, np_, kp, fp, 0, P.data_ptr(), stream())
    KD = torch.empty(fp.base.S * mp * np_, dtype=torch.int16, device="cuda")
    oztt.call("oztt_ii_digit_gemm", ga.data_ptr(), gb.data_ptr(), mp, np_, kp, fp, 1, KD.data_ptr(), stream())
    torch.cuda.synchronize()
    # oracle products over the padded planes (the padding digits are zero)
    ha = ga.view(fp.nplane, mp, kp).cpu().numpy()
    hb = gb.view(fp.nplane, np_, kp).cpu().numpy()
    bad, op = oracle.digit_gemm(np.ascontiguousarray(ha).reshape(-1), np.ascontiguousarray(hb).reshape(-1), fp, mp, np_,
                              kp)
    assert bad == 0
    assert np.array_equal(P.cpu().numpy(), op)
    # the fused composition: k_s = (sum_o coeff_o P_o) y_s mod m_s
    op = op.reshape(fp.nout, mp, np_).astype(np.int64)
    kd = KD.cpu().numpy().view(np.uint16).reshape(fp.base.S, mp, np_)
    r = oracle.digit_compose(np.ascontiguousarray(op.astype(np.int32)).reshape(-1), fp, crt, mp, np_).reshape(
        fp.base.S, mp, np_)
    for s in range(fp.base.S):
        mod = fp.base.moduli[s]
        acc = np.zeros((mp, np_), dtype=np.int64)
        for o in range(fp.oout[s], fp.oout[s + 1]):
            acc += (op[o] % mod) * fp.coeff[o]
        want = (acc % mod) * fp.base.yi[s] % mod
        assert np.array_equal(kd[s].astype(np.int64), want), f"modulus {s}"
        # the reference's binary32 composition gives the same residue class
        assert np.array_equal((r[s].astype(np.int64) * fp.base.yi[s]) % mod, want)


RUN_CASES = [(128, 128, 128, -1.0, 7, dict(reconstruction=1, fixed_bits=54)),
             (70, 130, 90, 0.5, 2, dict()),
             (64, 192, 64, 2.0, 4, dict(reconstruction=2)),
             (300, 200, 1000, 4.0, 9, dict(reconstruction=1, fixed_bits=64, max_moduli=16)),
             (96, 96, 600, 1.0, 12, dict(reconstruction=1, fixed_bits=99, max_moduli=24))]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,n,k,phi,seed,kw", RUN_CASES)
def test_pipeline_matches_oracle(oztt, oracle, cuda, m, n, k, phi, seed, kw, fmt):
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    fp, crt = plan_and_crt(oztt, oracle, a, b, m, n, k, fmt=fmt, **kw)
    c = oztt.digit_run(a, b, m, n, k, fp)
    rc, ce, err = oracle.digit_emulate(a, b, m, n, k, fp, exact=True)
    assert rc == 0, err
    assert np.array_equal(c.view(np.uint64), ce.view(np.uint64))
    rc, cf, err = oracle.digit_emulate(a, b, m, n, k, fp)
    assert rc == 0, err
    assert np.all(np.abs(c - cf).reshape(m, n) <= faithful_bound(oracle, a, b, m, n, k, crt, cf))
    hi, lo = oracle.dot2(a, b, m, n, k)
    rel, _ = oracle.accuracy(c, hi, lo)
    assert rel < 1e-15


PUBLISHED_128 = {FP8: "20046e5bb3816cbb", BF16: "13abe4ac7f292f42", FP16: "1811cf560959e61d",
                 TF32: "9a8f2780d4b9976b"}


@pytest.mark.parametrize("fmt", FORMATS)
def test_published_hash_on_gpu(oztt, oracle, cuda, fmt):
    """tools/validated/quick.csv:3,5,7,11: the GPU digit planes and products with the reference's composition
    and triple-float reconstruction restated on the host give every output bit of the reference device."""
    n = 128
    a, b, fp, crt, dA, dB, ga, gb, mp, np_, kp = digit_case(oztt, oracle, n, n, n, -1.0, 7,
                                                           dict(reconstruction=1, fixed_bits=54), fmt)
    P = torch.empty(fp.nout * mp * np_, dtype=torch.int32, device="cuda")
    oztt.call("oztt_ii_digit_gemm", ga.data_ptr(), gb.data_ptr(), mp, np_, kp, fp, 0, P.data_ptr(), stream())
    torch.cuda.synchronize()
    p = np.ascontiguousarray(P.view(fp.nout, mp, np_)[:, :n, :n].cpu().numpy())
    r = oracle.digit_compose(p.reshape(-1), fp, crt, n, n)
    c = oracle.recon_residue(r, n, n, dA.cpu().numpy(), dB.cpu().numpy(), crt)
    assert oracle.output_hash(c) == PUBLISHED_128[fmt]


PATTERNS = {"uniform": 0, "zero-A": 1, "nonnegative": 2, "scaled": 3, "cancellation": 4, "zero-row-column": 5,
            "smallest-maximum": 6, "largest-maximum": 7}
CHECKS = [(64, 64, 64, "uniform", 0), (3, 5, 7, "nonnegative", 0), (65, 67, 97, "scaled", 0), (9, 11, 17, "zero-A", 0),
          (3, 5, 64, "cancellation", 0), (3, 5, 7, "zero-row-column", 0), (1, 1, 1, "smallest-maximum", 0),
          (1, 1, 1, "largest-maximum", 0), (5056, 64, 32, "uniform", 0), (64, 64, 64, "uniform", 2)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,n,k,pattern,recon", CHECKS)
def test_correctness_cases(oztt, oracle, cuda, m, n, k, pattern, recon, fmt):
    """The acceptance cases of the reference's tests/correctness.cpp with each digit format (relative Frobenius
    error <= 8 eps against the compensated reference)."""
    a, b = oracle.gen_pattern(m, n, k, PATTERNS[pattern])
    c = np.full(m * n, 123.0)
    info = oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(format=fmt, reconstruction=recon))
    assert np.all(np.isfinite(c))
    hi, lo = oracle.dot2(a, b, m, n, k)
    rel, _ = oracle.accuracy(c, hi, lo)
    assert rel <= 8 * np.finfo(float).eps, rel
    assert info.format == fmt and info.scheme == oztt.Scheme.II
    assert info.padded_m == round_up(m, 64) and info.padded_n == round_up(n, 64) and info.padded_k == round_up(k, 32)
    assert info.moduli >= 2 and info.integer_bits >= 53
    if recon == 2:
        assert info.reconstruction_passes == 2


@pytest.mark.parametrize("fmt", FORMATS)
def test_context_matches_planned_run(oztt, oracle, cuda, fmt):
    """Context::gemm with a digit format plans on the device (statistics measured there) and gives the bits
    of the stage pipeline run with the host plan."""
    m, n, k = 300, 200, 500
    a, b = oracle.gen_inputs(m, n, k, 0.5, 21)
    fp = oztt.digit_plan(a, b, m, n, k, fmt=fmt)
    c = np.empty(m * n)
    info = oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(format=fmt))
    assert info.moduli == fp.base.S and info.integer_bits == fp.base.b
    c2 = oztt.digit_run(a, b, m, n, k, fp)
    assert np.array_equal(c.view(np.uint64), c2.view(np.uint64))
    A, B = dev(a), dev(b)
    fpd = oztt.digit_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, stream=stream(), fmt=fmt)
    assert bytes(fpd) == bytes(fp)
    C = torch.empty(m * n, dtype=torch.float64, device="cuda")
    ms = oztt.digit_run_device(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, fp, stream(), timed=True)
    assert len(ms) == 6 and all(x >= 0 for x in ms)
    assert np.array_equal(C.cpu().numpy().view(np.uint64), c.view(np.uint64))


@pytest.mark.parametrize("fmt", FORMATS)
def test_context_streamed_bands(oztt, oracle, cuda, fmt):
    """Context::gemm's streamed path with a digit format: B in two blocks of columns, A in three blocks of
    columns (the last one ragged), two row bands (the last one ragged), tiny elements in both operands (the
    statistics' scale-first recomputation); the bits of the stage pipeline run with the host plan."""
    m, n, k = 4500, 2048, 4608
    a, b = oracle.gen_inputs(m, n, k, 1.0, 23)
    a[11], b[k * n - 3] = 2.0 ** -500, -(2.0 ** -420)
    fp = oztt.digit_plan(a, b, m, n, k, fmt=fmt)
    c = np.full(m * n, 123.0)
    info = oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(format=fmt))
    assert info.moduli == fp.base.S and info.integer_bits == fp.base.b
    c2 = oztt.digit_run(a, b, m, n, k, fp)
    assert np.array_equal(c.view(np.uint64), c2.view(np.uint64))
    assert oztt.ii_int8_last_phases()["bands"] == 2


@pytest.mark.parametrize("fmt", FORMATS)
def test_context_streamed_check_errors(oztt, cuda, fmt):
    """A value error is reported from the measured maxima in the reference's order, before any plan
    error, with C untouched."""
    ctx = oztt.Context()
    m = n = k = 200
    rng = np.random.default_rng(3)
    a = rng.standard_normal(m * k)
    b = rng.standard_normal(k * n)
    c = np.full(m * n, 123.0)
    b[7] = np.inf
    with pytest.raises(ValueError, match="B contains NaN or infinity"):
        ctx.gemm(a, b, c, m, n, k, oztt.Options(format=fmt, max_moduli=2))
    b[7] = 1.0
    with pytest.raises(ValueError, match="must be in"):  # a row of A whose maximum is below 2^-126
        ctx.gemm(np.full(k, 2.0 ** -140), b, c[:n], 1, n, k, oztt.Options(format=fmt))
    assert np.all(c == 123.0)


def test_rejections(oztt, cuda):
    ctx = oztt.Context()
    a = np.ones(64 * 64)
    c = np.full(64 * 64, 123.0)
    with pytest.raises(RuntimeError):
        ctx.gemm(a, a, c, 64, 64, 64, oztt.Options(format=oztt.Format.FP8, max_moduli=2))
    assert np.all(c == 123.0)
    buf = np.array([1.0, 2.0, 3.0, 4.0])
    ctx.gemm(buf, np.array([1.0, 0.0, 0.0, 1.0]), buf, 2, 2, 2, oztt.Options(format=oztt.Format.FP8))
    assert buf.tolist() == [1.0, 2.0, 3.0, 4.0]
