"""Scheme II INT8 on the B200, stage by stage and end to end, against the oracle.

Every call goes through the C ABI of liboztt.so. Bars:
  * scale (BF16 maxima, exponent deltas, range flags), residue planes, C_s (int32) and the CRT digits:
    bit-exact;
  * the FP64 output: bit-exact against the oracle's restatement of the B200 exact CRT, and within the
    componentwise tolerance |C - C_ref| <= 2^-65 * KM * 2^(2 shift - dA_i - dB_j) + 2 ulp(C_ref) of the
    reference's own (triple-float) reconstruction;
  * the acceptance cases of the reference's tests/correctness.cpp: relative Frobenius error <= 8 eps
    against a compensated (Dot2) reference.
"""

import numpy as np
import pytest
import torch

from oracle_lib import pad, round_up

pytestmark = pytest.mark.gpu


def dev(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return t.cuda() if dtype is None else t.to(dtype).cuda()


def stream():
    return torch.cuda.current_stream().cuda_stream


def plan_for(oztt, a, b, m, n, k, **kw):
    return oztt.ii_int8_plan(a, b, m, n, k, **kw)


def oracle_plan(oracle, a, b, m, n, k, fixed_bits=0, passes=0, max_moduli=0):
    M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
    rc, p, err = oracle.plan(pad(a, m, k, M, K), pad(b, k, n, K, N), M, N, K, max_moduli, passes, fixed_bits)
    assert rc == 0, err
    return p


def gpu_scale(oztt, x, rows, cols, col_mode, shift):
    X = dev(x)
    nout = cols if col_mode else rows
    delta = torch.zeros(nout, dtype=torch.int32, device="cuda")
    bf = torch.zeros(nout, dtype=torch.int16, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    name = "oztt_ii_scale_cols" if col_mode else "oztt_ii_scale_rows"
    oztt.call(name, X.data_ptr(), rows, cols, cols, shift, delta.data_ptr(), bf.data_ptr(), flags.data_ptr(), stream())
    torch.cuda.synchronize()
    return bf.cpu().numpy().view(np.uint16), delta.cpu().numpy(), int(flags.cpu().numpy()[0])


SCALE_CASES = [(64, 64, -1.0), (33, 100, 0.5), (257, 129, 4.0), (1000, 3, 8.0), (7, 4097, 1.0)]


@pytest.mark.parametrize("m,k,phi", SCALE_CASES)
def test_scale_matches_oracle(oztt, oracle, cuda, m, k, phi):
    a, b = oracle.gen_inputs(m, k, k, phi, 3)
    for col_mode, x, rows, cols in ((0, a, m, k), (1, b, k, k)):
        bf, d, fl = gpu_scale(oztt, x, rows, cols, col_mode, 14)
        obf, od, ofl = oracle.scale(x, rows, cols, col_mode, 14)
        assert np.array_equal(bf, obf) and np.array_equal(d, od) and fl == ofl


def test_scale_edge_rows(oztt, oracle, cuda):
    """Zero rows, exact powers of two, maxima at both ends of the BF16 range, and the range flags."""
    rows = [np.zeros(9), np.full(9, 0.5), np.full(9, 2.0 ** -126), np.full(9, float.fromhex('0x1.fep127')), np.full(9, 2.0 ** -130),
            np.full(9, 2.0 ** 128), np.array([1.0] * 8 + [np.inf]), np.array([1.0] * 8 + [np.nan]),
            np.array([-3.0, 1e-300, 0, 0, 0, 0, 0, 0, 5e-324]), np.array([float.fromhex('0x1.0000000000001p0')] + [0.0] * 8)]
    x = np.concatenate(rows)
    for r in range(len(rows)):
        bf, d, fl = gpu_scale(oztt, x[9 * r:9 * r + 9], 1, 9, 0, 14)
        obf, od, ofl = oracle.scale(x[9 * r:9 * r + 9].copy(), 1, 9, 0, 14)
        assert (bf[0], d[0], fl) == (obf[0], od[0], ofl), r
    # columns mode on the transposed rows
    xt = np.ascontiguousarray(x.reshape(len(rows), 9).T).reshape(-1)
    bf, d, fl = gpu_scale(oztt, xt, 9, len(rows), 1, 14)
    obf, od, ofl = oracle.scale(xt, 9, len(rows), 1, 14)
    assert np.array_equal(bf, obf) and np.array_equal(d, od) and fl == ofl == 7


def gpu_split(oztt, x, rows, cols, col_mode, delta, plan):
    mp, np_, kp = oztt.padded_dims(rows if not col_mode else 1, cols if col_mode else 1, cols if not col_mode else rows)
    X = dev(x)
    D = dev(delta.astype(np.int32))
    if col_mode:  # B: rows = K, cols = N -> planes [S][np][kp]
        planes = torch.zeros(plan.S * np_ * kp, dtype=torch.int8, device="cuda")
        oztt.call("oztt_ii_split_cols", X.data_ptr(), rows, cols, cols, D.data_ptr(), plan, planes.data_ptr(), np_, kp,
                  stream())
        shape = (plan.S, np_, kp)
    else:
        planes = torch.zeros(plan.S * mp * kp, dtype=torch.int8, device="cuda")
        oztt.call("oztt_ii_split_rows", X.data_ptr(), rows, cols, cols, D.data_ptr(), plan, planes.data_ptr(), mp, kp,
                  stream())
        shape = (plan.S, mp, kp)
    torch.cuda.synchronize()
    return planes.cpu().numpy().reshape(shape)


# widths 54-56, 61 and 81 leave the top digit below 2^16 (kept whole by the odd-modulus residues); 58, 77 and
# 100 put it above (split into halves)
SPLIT_CASES = [(64, 64, 64, -1.0, 54), (70, 90, 130, 0.5, 56), (128, 64, 300, 4.0, 61), (33, 65, 200, 8.0, 81),
               (256, 256, 256, 2.0, 100), (96, 80, 160, 1.0, 58), (40, 48, 96, 2.0, 77)]


@pytest.mark.parametrize("m,n,k,phi,bfix", SPLIT_CASES)
def test_split_matches_oracle(oztt, oracle, cuda, m, n, k, phi, bfix):
    a, b = oracle.gen_inputs(m, n, k, phi, 5)
    plan = plan_for(oztt, a, b, m, n, k, fixed_bits=bfix, reconstruction=1, max_moduli=24)
    op = oracle_plan(oracle, a, b, m, n, k, fixed_bits=bfix, passes=1, max_moduli=24)
    assert plan.moduli_list == op.moduli and plan.nd == op.nd
    _, dA, _ = oracle.scale(a, m, k, 0, plan.shift)
    _, dB, _ = oracle.scale(b, k, n, 1, plan.shift)
    ga = gpu_split(oztt, a, m, k, 0, dA, plan)
    gb = gpu_split(oztt, b, k, n, 1, dB, plan)
    S = plan.S
    mp, np_, kp = ga.shape[1], gb.shape[1], ga.shape[2]
    ap = pad(a, m, k, mp, kp)
    oa = oracle.split(ap, mp, kp, 0, np.concatenate([dA, np.zeros(mp - m, np.int32)]), op).reshape(S, mp, kp)
    bp = pad(b, k, n, kp, np_)
    ob = oracle.split(bp, kp, np_, 1, np.concatenate([dB, np.zeros(np_ - n, np.int32)]), op).reshape(S, np_, kp)
    assert np.array_equal(ga, oa), f"A residues differ at {np.argwhere(ga != oa)[:5]}"
    assert np.array_equal(gb, ob), f"B residues differ at {np.argwhere(gb != ob)[:5]}"
    assert np.abs(ga).max() <= 127 and not ga[:, m:, :].any() and not ga[:, :, k:].any()


@pytest.mark.parametrize("bits", [54, 58])
def test_split_hard_elements(oztt, oracle, cuda, bits):
    """Elements that stress the triple-float split: ties of the 30-bit rounding, long runs of ones,
    values far below the row maximum, subnormals, exact powers of two and the m=254 tie residues (top
    digit whole at 54 bits, split at 58)."""
    rng = np.random.default_rng(11)
    k = 512
    vals = []
    for _ in range(k):
        x = float(rng.uniform(0.5, 1.0)) * 2.0 ** int(rng.integers(-80, 1))
        bits = np.frombuffer(np.float64(x).tobytes(), np.uint64)[0]
        kind = rng.integers(0, 5)
        if kind == 0:
            bits = (bits & ~np.uint64(0x3FFFFFFF)) | np.uint64(0x20000000)
        elif kind == 1:
            bits = bits | np.uint64(0xFFFFFFF)
        elif kind == 2:
            bits = (bits & ~np.uint64(0x3FFFFFFF)) | np.uint64(0x20000000 + int(rng.integers(1, 127)))
        x = float(np.frombuffer(np.uint64(bits).tobytes(), np.float64)[0])
        vals.append(-x if rng.integers(0, 2) else x)
    vals[:8] = [1.0, -1.0, 0.5, 2.0 ** -100, 5e-324, 2.0 ** -1022, 0.0, -0.0]
    a = np.array(vals * 64)  # 64 rows of the same pattern with different row maxima
    for r in range(64):
        a[r * k] = 2.0 ** (r - 32)
    m = 64
    b = np.ones(k * 64)
    plan = plan_for(oztt, a, b, m, 64, k, fixed_bits=bits, reconstruction=1)
    op = oracle_plan(oracle, a, b, m, 64, k, fixed_bits=bits, passes=1)
    _, dA, _ = oracle.scale(a, m, k, 0, plan.shift)
    ga = gpu_split(oztt, a, m, k, 0, dA, plan)
    mp, kp = ga.shape[1], ga.shape[2]
    oa = oracle.split(pad(a, m, k, mp, kp), mp, kp, 0, np.concatenate([dA, np.zeros(mp - m, np.int32)]),
                      op).reshape(plan.S, mp, kp)
    assert np.array_equal(ga, oa)


def gpu_residue_gemm(oztt, ra, rb, mp, np_, kp, plan, mode):
    A = dev(ra.reshape(-1))
    B = dev(rb.reshape(-1))
    dtype = torch.int32 if mode == 0 else torch.uint8
    out = torch.full((plan.S * mp * np_,), 77, dtype=dtype, device="cuda")
    oztt.call("oztt_ii_residue_gemm", A.data_ptr(), B.data_ptr(), mp, np_, kp, plan, mode, out.data_ptr(), stream())
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(plan.S, mp, np_)


GEMM_CASES = [(128, 256, 128, 54), (256, 512, 384, 54), (384, 256, 1024, 56), (128, 768, 2048, 61)]


@pytest.mark.parametrize("mp,np_,kp,bfix", GEMM_CASES)
def test_residue_gemm_matches_oracle(oztt, oracle, cuda, mp, np_, kp, bfix):
    rng = np.random.default_rng(mp + np_ + kp)
    a = rng.uniform(-1, 1, mp * kp)
    b = rng.uniform(-1, 1, kp * np_)
    plan = plan_for(oztt, a, b, mp, np_, kp, fixed_bits=bfix, reconstruction=1)
    S = plan.S
    ra = rng.integers(-127, 128, (S, mp, kp), dtype=np.int8)
    rb = rng.integers(-127, 128, (S, np_, kp), dtype=np.int8)
    ra[:, :3, :] = 127  # extreme sums
    rb[:, :3, :] = 127
    rb[:, 3:6, :] = -127
    c32 = gpu_residue_gemm(oztt, ra, rb, mp, np_, kp, plan, 0)
    want = oracle.gemm_i32(ra.reshape(-1), rb.reshape(-1), S, mp, np_, kp).reshape(S, mp, np_)
    assert np.array_equal(c32, want), f"C_s differs at {np.argwhere(c32 != want)[:5]}"
    k8 = gpu_residue_gemm(oztt, ra, rb, mp, np_, kp, plan, 1)
    m = np.array(plan.moduli_list, dtype=np.int64)[:, None, None]
    y = np.array([plan.yi[i] for i in range(S)], dtype=np.int64)[:, None, None]
    kk = ((want.astype(np.int64) % m) * y) % m
    assert np.array_equal(k8.astype(np.int64), kk)


def test_residue_gemm_large_vs_cublas(oztt, cuda):
    """A full-size tile grid (several waves of the persistent kernel) checked against an exact int8
    GEMM from torch for two moduli."""
    mp, np_, kp = 2048, 2048, 4096
    a = np.ones(2)
    plan = plan_for(oztt, a, a, 2, 2, 1, fixed_bits=54, reconstruction=1, max_moduli=16)
    S = plan.S
    g = torch.Generator(device="cuda").manual_seed(1)
    A = torch.randint(-127, 128, (S, mp, kp), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-127, 128, (S, np_, kp), dtype=torch.int8, device="cuda", generator=g)
    out = torch.zeros((S, mp, np_), dtype=torch.int32, device="cuda")
    oztt.call("oztt_ii_residue_gemm", A.data_ptr(), B.data_ptr(), mp, np_, kp, plan, 0, out.data_ptr(), stream())
    torch.cuda.synchronize()
    for s in (0, S - 1):
        ref = torch._int_mm(A[s], B[s].t())
        assert torch.equal(out[s], ref)


RECON_CASES = [(64, 64, 64, -1.0, 54, 1), (130, 70, 90, 0.5, 56, 2), (96, 300, 128, 4.0, 61, 1),
               (64, 64, 256, 8.0, 81, 1), (200, 100, 64, 1.0, 100, 2)]


@pytest.mark.parametrize("m,n,k,phi,bfix,passes", RECON_CASES)
def test_pipeline_matches_oracle(oztt, oracle, cuda, m, n, k, phi, bfix, passes):
    a, b = oracle.gen_inputs(m, n, k, phi, 13)
    plan = plan_for(oztt, a, b, m, n, k, fixed_bits=bfix, reconstruction=passes, max_moduli=24)
    c = oztt.ii_int8_run(a, b, m, n, k, plan)
    rc, cx, op, err = oracle.emulate(a, b, m, n, k, max_moduli=24, passes=passes, fixed_bits=bfix, exact=True)
    assert rc == 0, err
    assert op.moduli == plan.moduli_list
    assert np.array_equal(c.view(np.uint64), cx.view(np.uint64)), "differs from the exact CRT restated on the CPU"
    rc, cf, _, _ = oracle.emulate(a, b, m, n, k, max_moduli=24, passes=passes, fixed_bits=bfix, exact=False)
    M, N = round_up(m, 64), round_up(n, 64)
    K = round_up(k, 32)
    _, dA, _ = oracle.scale(pad(a, m, k, M, K), M, K, 0, plan.shift)
    _, dB, _ = oracle.scale(pad(b, k, n, K, N), K, N, 1, plan.shift)
    KM = (op.W_hi * 2.0 ** 32 + op.W_lo) * 2.0 ** op.qw
    g = 2 * plan.shift - (dA[:m, None] + dB[None, :n])
    tol = (2.0 ** -90 if passes == 2 else 2.0 ** -65) * KM * np.exp2(g.astype(np.float64))
    bound = tol + 2 * np.spacing(np.abs(cf.reshape(m, n)))
    assert np.all(np.abs(c.reshape(m, n) - cf.reshape(m, n)) <= bound)


def test_published_case_on_gpu(oztt, oracle, cuda):
    """The published case of tools/validated/quick.csv:13 (n=128, seed 7, b=54): C within the
    reference tolerance of the reference output (hash fe063f5214e93e2e), same moduli, same accuracy."""
    n = 128
    a, b = oracle.gen_inputs(n, n, n, -1.0, 7)
    plan = plan_for(oztt, a, b, n, n, n, fixed_bits=54)
    assert plan.S == 15 and plan.two_pass == 0
    c = oztt.ii_int8_run(a, b, n, n, n, plan)
    rc, cf, op, _ = oracle.emulate(a, b, n, n, n, fixed_bits=54)
    assert oracle.output_hash(cf) == "fe063f5214e93e2e"
    hi, lo = oracle.dot2(a, b, n, n, n)
    rel_gpu, bits_gpu = oracle.accuracy(c, hi, lo)
    rel_ref, _ = oracle.accuracy(cf, hi, lo)
    assert rel_gpu <= rel_ref * 1.0000001 and bits_gpu > 54.2
    assert np.max(np.abs(c - cf)) <= 2.0 ** -50 * np.max(np.abs(cf))


# ---- acceptance cases of the reference's tests/correctness.cpp:174-237 ------------------------------
PATTERNS = {"uniform": 0, "zero-A": 1, "nonnegative": 2, "scaled": 3, "cancellation": 4, "zero-row-column": 5,
            "smallest-maximum": 6, "largest-maximum": 7}
CHECKS = [(64, 64, 64, "uniform", 0), (3, 5, 7, "nonnegative", 0), (65, 67, 97, "scaled", 0), (9, 11, 17, "zero-A", 0),
          (3, 5, 64, "cancellation", 0), (3, 5, 7, "zero-row-column", 0), (1, 1, 1, "smallest-maximum", 0),
          (1, 1, 1, "largest-maximum", 0), (5056, 64, 32, "uniform", 0), (64, 64, 64, "uniform", 2)]


@pytest.mark.parametrize("m,n,k,pattern,recon", CHECKS)
def test_correctness_cases(oztt, oracle, cuda, m, n, k, pattern, recon):
    a, b = oracle.gen_pattern(m, n, k, PATTERNS[pattern])
    c = np.full(m * n, 123.0)
    info = oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(format=oztt.Format.INT8, reconstruction=recon))
    assert np.all(np.isfinite(c))
    hi, lo = oracle.dot2(a, b, m, n, k)
    rel, _ = oracle.accuracy(c, hi, lo)
    assert rel <= 8 * np.finfo(float).eps, rel
    assert info.padded_m == round_up(m, 64) and info.padded_n == round_up(n, 64) and info.padded_k == round_up(k, 32)
    assert info.moduli >= 2 and info.integer_bits >= 53
    if recon == 2:
        assert info.reconstruction_passes == 2


def test_overlap_and_rejection(oztt, cuda):
    ctx = oztt.Context()
    opt = oztt.Options(format=oztt.Format.INT8)
    buf = np.array([1.0, 2.0, 3.0, 4.0])
    ctx.gemm(buf, np.array([1.0, 0.0, 0.0, 1.0]), buf, 2, 2, 2, opt)  # C aliases A
    assert buf.tolist() == [1.0, 2.0, 3.0, 4.0]
    a = np.ones(64 * 64)
    c = np.full(64 * 64, 123.0)
    with pytest.raises(RuntimeError):
        ctx.gemm(a, a, c, 64, 64, 64, oztt.Options(format=oztt.Format.INT8, max_moduli=2))
    assert np.all(c == 123.0)
    assert ctx.multiply([1, 2, 3, 4, 5, 6], [7, 8, 9, 10, 11, 12], 2, 2, 3, opt).tolist() == [58, 64, 139, 154]


def test_device_run_matches_host_run(oztt, oracle, cuda):
    m, n, k = 300, 200, 500
    a, b = oracle.gen_inputs(m, n, k, 0.5, 21)
    plan = plan_for(oztt, a, b, m, n, k)
    c_host = oztt.ii_int8_run(a, b, m, n, k, plan)
    A, B = dev(a), dev(b)
    C = torch.empty(m * n, dtype=torch.float64, device="cuda")
    oztt.ii_int8_run_device(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, plan, stream())
    assert np.array_equal(C.cpu().numpy().view(np.uint64), c_host.view(np.uint64))
    # repeated calls give the same bits
    oztt.ii_int8_run_device(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, plan, stream())
    assert np.array_equal(C.cpu().numpy().view(np.uint64), c_host.view(np.uint64))


# ---- Context.gemm's streamed path: chunked upload, statistics as chunks land, banded read-back ----------
# Sizes: 4096 rows and more compute while their operands upload (A's first half, B in blocks of about n/8
# columns, the rest of A in bands of 1024 rows, B's last blocks): (9000, 256, 256) one block of B, a ragged last band;
# (4500, 4608, 2048) six blocks of B (the last one ragged). Below 4096 rows B and A go up in blocks of
# max(512, 64 MiB / 8k) and max(512, 64 MiB / 8m) columns, then row bands of about 2048 rows (up to 8):
# (3000, 2048, 4608) two column blocks of B and of A, with tiny elements (below 2^-383) in both operands.
@pytest.mark.parametrize("m,n,k,phi,seed", [(9000, 256, 256, 0.5, 31), (4500, 4608, 2048, 1.0, 32),
                                            (3000, 2048, 4608, 1.0, 33)])
def test_context_streamed_matches_planned_run(oztt, oracle, cuda, m, n, k, phi, seed):
    a, b = oracle.gen_inputs(m, n, k, phi, seed)
    if seed == 33:
        a[7], a[m * k // 2] = 2.0 ** -600, -5e-324
        b[k * n - 5] = 2.0 ** -450
    plan = plan_for(oztt, a, b, m, n, k)  # host statistics
    c_ref = oztt.ii_int8_run(a, b, m, n, k, plan)
    c = np.full(m * n, 123.0)
    info = oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(format=oztt.Format.INT8))
    assert info.moduli == plan.S and info.integer_bits == plan.b
    assert info.reconstruction_passes == (2 if plan.two_pass else 1)
    assert np.array_equal(c.view(np.uint64), c_ref.view(np.uint64))
    ph = oztt.ii_int8_last_phases()
    assert ph["bands"] == expected_bands(m, n)
    assert ph["total_ms"] > 0 and ph["upload_ms"] > 0


def expected_bands(m, n):
    mp = round_up(m, 128)
    if mp >= 4096:  # the path that computes while its operands upload: A's first half against each of B's
        pre = min(round_up(m // 2, 1024), m)  # first blocks (one tile each), each later band of 1024 rows (one
        nb = round_up(-(-n // 8), 256)        # tile), then each of B's last blocks against the whole A in parts
        nblocks = -(-n // nb)                 # of 4096 rows (the last block: 2048)
        first = min(nblocks // 2, nblocks - 1) + 1
        last = sum(-(-m // (4096 if j + 1 < nblocks else 2048)) for j in range(first, nblocks))
        return first + -(-(m - pre) // 1024) + last
    bm = round_up(-(-mp // min(8, max(1, mp // 2048))), 128)
    return -(-mp // bm)


def test_context_streamed_reports_check_errors_first(oztt, cuda):
    """A value error found by the host checks that run during the upload is the error reported, and C
    stays untouched, also when the plan would fail (max_moduli = 2)."""
    ctx = oztt.Context()
    m = n = k = 300
    rng = np.random.default_rng(5)
    a = rng.standard_normal(m * k)
    b = rng.standard_normal(k * n)
    a[m * k - 1] = np.nan
    c = np.full(m * n, 123.0)
    for opt in (oztt.Options(format=oztt.Format.INT8), oztt.Options(format=oztt.Format.INT8, max_moduli=2)):
        with pytest.raises(ValueError, match="A contains NaN or infinity"):
            ctx.gemm(a, b, c, m, n, k, opt)
    a[m * k - 1] = 1.0
    b[5] = 2.0 ** 130
    with pytest.raises(ValueError, match="must be in"):
        ctx.gemm(a, b, c, m, n, k, oztt.Options(format=oztt.Format.INT8))
    assert np.all(c == 123.0)
    # a valid call afterwards runs normally
    b[5] = 1.0
    ctx.gemm(a, b, c, m, n, k, oztt.Options(format=oztt.Format.INT8))
    assert np.all(np.isfinite(c))
