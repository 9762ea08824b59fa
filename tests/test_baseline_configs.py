"""The BASELINE configurations pinned against the reference's own planners, and configs 1 and 2 run
end to end on the GPU against the oracle.

tests/golden/baseline_plans.json holds the decisions of the reference's planner code compiled in place
(tests/golden/make_baseline_plans.py) on the BASELINE inputs: the evaluator's generator
(evaluation/numerics.hpp:19-38, mt19937 seed 0, (u - 1/2) exp(phi z)) at
  config 1   Scheme II INT8 256^3, phi 0.5, auto precision, Automatic reconstruction
  config 2   Scheme II INT8 4096^3, phi 0.5, auto precision, TwoPass
  config 3   Scheme I INT8 8192^3, phi 1.0, slice count selected from the input
  config 4   Scheme II FP8 / BF16 8192 x 8192 x 16384, phi 4.0, max_moduli 12/16/20/24 x one/two passes
  metric     Scheme II INT8 16384^3, phi 0.5, auto precision (the headline bench point)
Every plan this library makes for those inputs -- on the host (CPU tests, the sizes the CPU suite affords)
and from the device-measured statistics that Context::gemm uses (GPU tests, every size) -- must take the
reference's decisions: the same accept/reject, moduli, width, passes and, bit for bit, the five input
statistics of the precision policy.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle_lib import pad, round_up

GOLDEN = {c["name"]: c for c in json.loads((Path(__file__).parent / "golden" / "baseline_plans.json").read_text())
          ["cases"]}
FMT = {"FP8": 4, "BF16": 0}


def _hexs(vals):
    return [float.hex(float(v)) for v in vals]


def _check_ii(plan, case):
    assert case["rc"] == 0
    assert (plan.S, plan.b, plan.two_pass, plan.moduli_list, plan.b_cap) == \
           (case["S"], case["b"], case["two_pass"], case["moduli"], case["b_cap"])
    assert _hexs((plan.TA, plan.TB, plan.nA, plan.nB, plan.nC)) == case["stats"]


def _inputs(oracle, case):
    return oracle.gen_inputs(case["m"], case["n"], case["k"], case["phi"], case["seed"])


# ---- host planner (CPU) ------------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["config1", "config2"])
def test_host_plan_equals_reference(oztt, oracle, name):
    case = GOLDEN[name]
    a, b = _inputs(oracle, case)
    plan = oztt.ii_int8_plan(a, b, case["m"], case["n"], case["k"], case["max_moduli"], case["passes"],
                             case["fixed_bits"])
    _check_ii(plan, case)


def test_oracle_plan_equals_reference_config1(oracle):
    case = GOLDEN["config1"]
    a, b = _inputs(oracle, case)
    n = case["m"]
    rc, p, err = oracle.plan(a, b, n, n, n, 0, 0, 0)
    assert rc == 0, err
    assert (p.S, p.b, p.two_pass, p.moduli) == (case["S"], case["b"], case["two_pass"], case["moduli"])


def test_fixture_matches_the_survey_predictions():
    """The survey's probe of the reference planner: config 1 -> b = 55, S = 16, one pass; config 2 -> b = 56,
    S = 16; config 4 FP8 with max_moduli 12 rejected (48 bits), BF16 with 20 rejected; the metric point takes
    b = 56."""
    assert (GOLDEN["config1"]["b"], GOLDEN["config1"]["S"], GOLDEN["config1"]["two_pass"]) == (55, 16, 0)
    assert (GOLDEN["config2"]["b"], GOLDEN["config2"]["S"]) == (56, 16)
    assert GOLDEN["config4-FP8-S12-p1"]["rc"] == 1
    assert GOLDEN["config4-BF16-S20-p1"]["rc"] == 1
    assert GOLDEN["metric"]["rc"] == 0 and GOLDEN["metric"]["b"] == 56


# ---- device-measured plans (GPU) ---------------------------------------------------------------------
def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["config1", "config2", "metric"])
def test_device_plan_equals_reference_int8(oztt, oracle, cuda, name):
    import torch

    case = GOLDEN[name]
    a, b = _inputs(oracle, case)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    del a, b
    plan = oztt.ii_int8_plan_device(A.data_ptr(), B.data_ptr(), case["m"], case["n"], case["k"],
                                    max_moduli=case["max_moduli"], reconstruction=case["passes"],
                                    fixed_bits=case["fixed_bits"], stream=_stream())
    _check_ii(plan, case)


@pytest.mark.gpu
def test_device_plans_equal_reference_config4(oztt, oracle, cuda):
    import torch

    first = GOLDEN["config4-FP8-S12-p1"]
    a, b = _inputs(oracle, first)
    m, n, k = first["m"], first["n"], first["k"]
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    del a, b
    bad = []
    for name, case in GOLDEN.items():
        if not name.startswith("config4-"):
            continue
        try:
            p = oztt.digit_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, max_moduli=case["max_moduli"],
                                       reconstruction=case["passes"], stream=_stream(),
                                       fmt=oztt.Format(FMT[case["format"]]))
            rc = 0
        except (RuntimeError, ValueError):
            p, rc = None, 1
        if rc != case["rc"]:
            bad.append((name, "rc", rc))
            continue
        if p is None:
            continue
        got = (p.base.S, p.base.b, p.base.two_pass, [int(p.base.moduli[i]) for i in range(p.base.S)], p.nplane,
               p.nprod, p.nout, _hexs((p.base.TA, p.base.TB, p.base.nA, p.base.nB, p.base.nC)))
        want = (case["S"], case["b"], case["two_pass"], case["moduli"], case["nplane"], case["nprod"], case["nout"],
                case["stats"])
        if got != want:
            bad.append((name, got, want))
    assert not bad, bad


@pytest.mark.gpu
def test_scheme_i_slices_equal_reference_config3(oztt, oracle, cuda):
    import torch

    case = GOLDEN["config3-auto"]
    a, b = _inputs(oracle, case)
    m, n, k = case["m"], case["n"], case["k"]
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    plan = oztt.i_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, slices=0, stream=_stream())
    assert plan.p == case["p"] and plan.auto_p == 1
    # the fixed sweep of the configuration: every p in 4..12 is executable at K = 8192 (the INT8 Horner
    # budget of ozaki1/format.hpp allows p <= 12 there)
    for p in range(4, 13):
        assert oztt.i_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, slices=p, stream=_stream()).p == p


# ---- configs 1 and 2 end to end (GPU) ------------------------------------------------------------------
def _tolerance(op, plan, dA, dB, passes):
    """|C - C_ref| bound of the reference's own triple-float reconstruction, componentwise."""
    KM = (op.W_hi * 2.0 ** 32 + op.W_lo) * 2.0 ** op.qw
    g = 2 * plan.shift - (dA[:, None].astype(np.int64) + dB[None, :].astype(np.int64))
    return (2.0 ** -90 if passes == 2 else 2.0 ** -65) * KM * np.exp2(g.astype(np.float64))


@pytest.mark.gpu
def test_config1_end_to_end(oztt, oracle, cuda):
    case = GOLDEN["config1"]
    a, b = _inputs(oracle, case)
    n = case["m"]
    c = np.empty(n * n)
    info = oztt.Context().gemm(a, b, c, n, n, n, oztt.Options(format=oztt.Format.INT8))
    assert (info.moduli, info.integer_bits, info.reconstruction_passes) == (case["S"], case["b"], 1)
    rc, cx, op, err = oracle.emulate(a, b, n, n, n, exact=True)
    assert rc == 0, err
    assert op.moduli == case["moduli"]
    assert np.array_equal(c.view(np.uint64), cx.view(np.uint64)), "differs from the exact CRT restated on the CPU"
    rc, cf, _, _ = oracle.emulate(a, b, n, n, n, exact=False)
    _, dA, _ = oracle.scale(a, n, n, 0, op.shift)
    _, dB, _ = oracle.scale(b, n, n, 1, op.shift)
    bound = _tolerance(op, op, dA, dB, 1) + 2 * np.spacing(np.abs(cf.reshape(n, n)))
    assert np.all(np.abs(c.reshape(n, n) - cf.reshape(n, n)) <= bound)
    # the accuracy criterion: no worse than twice the reference's own result against binary128
    e_b200, e_ref = oracle.maxrel_f128_rows(a, b, [c, cf], n, n, n, np.arange(n))
    assert e_b200 <= 2 * e_ref, (e_b200, e_ref)


@pytest.mark.gpu
def test_config2_stages_and_result(oztt, oracle, cuda):
    """4096^3 with TwoPass: the plan from the device statistics is the reference's; on sampled rows of A
    and columns of B the residue planes equal the oracle's, C_s equals the exact integer products of those
    planes, and C equals the exact CRT bit for bit and the reference's reconstruction within its
    two-pass tolerance; the whole C matches the pipeline run through Context::gemm."""
    import torch

    case = GOLDEN["config2"]
    n = case["m"]
    a, b = _inputs(oracle, case)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    st = _stream()
    plan = oztt.ii_int8_plan_device(A.data_ptr(), B.data_ptr(), n, n, n, reconstruction=2, stream=st)
    _check_ii(plan, case)
    S = plan.S
    mp, np_, kp = oztt.padded_dims(n, n, n)
    dA = torch.zeros(mp, dtype=torch.int32, device="cuda")
    dB = torch.zeros(np_, dtype=torch.int32, device="cuda")
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    oztt.call("oztt_ii_scale_rows", A.data_ptr(), n, n, n, plan.shift, dA.data_ptr(), None, flags.data_ptr(), st)
    oztt.call("oztt_ii_scale_cols", B.data_ptr(), n, n, n, plan.shift, dB.data_ptr(), None, flags[1:].data_ptr(), st)
    ra = torch.zeros(S * mp * kp, dtype=torch.int8, device="cuda")
    rb = torch.zeros(S * np_ * kp, dtype=torch.int8, device="cuda")
    oztt.call("oztt_ii_split_rows", A.data_ptr(), n, n, n, dA.data_ptr(), plan, ra.data_ptr(), mp, kp, st)
    oztt.call("oztt_ii_split_cols", B.data_ptr(), n, n, n, dB.data_ptr(), plan, rb.data_ptr(), np_, kp, st)
    cs = torch.empty(S * mp * np_, dtype=torch.int32, device="cuda")
    oztt.call("oztt_ii_residue_gemm", ra.data_ptr(), rb.data_ptr(), mp, np_, kp, plan, 0, cs.data_ptr(), st)
    C = torch.empty(n * n, dtype=torch.float64, device="cuda")
    oztt.ii_int8_run_device(A.data_ptr(), B.data_ptr(), C.data_ptr(), n, n, n, plan, stream=st)
    torch.cuda.synchronize()
    assert not flags.any()
    op = oracle.crt_plan(plan.moduli_list, plan.b, plan.two_pass)
    rows = np.array([0, 1, 777, 2048, 3001, n - 1])
    cols = np.array([0, 5, 1023, 2222, 4000, n - 1])
    dA_h, dB_h = dA.cpu().numpy()[:n], dB.cpu().numpy()[:n]
    # residues of the sampled rows of A and columns of B
    ra_h = ra.view(S, mp, kp)[:, torch.as_tensor(rows), :n].cpu().numpy()
    want_a = oracle.split(np.ascontiguousarray(a.reshape(n, n)[rows]).reshape(-1), len(rows), n, 0,
                          np.ascontiguousarray(dA_h[rows]), op).reshape(S, len(rows), n)
    assert np.array_equal(ra_h, want_a)
    rb_h = rb.view(S, np_, kp)[:, torch.as_tensor(cols), :n].cpu().numpy()
    want_b = oracle.split(np.ascontiguousarray(b.reshape(n, n)[:, cols]).reshape(-1), n, len(cols), 1,
                          np.ascontiguousarray(dB_h[cols]), op).reshape(S, len(cols), n)
    assert np.array_equal(rb_h, want_b)
    # C_s on the sampled rows (all columns): exact integer products of the planes
    rb_all = rb.view(S, np_, kp)[:, :n, :n].contiguous().cpu().numpy()
    cs_rows = cs.view(S, mp, np_)[:, torch.as_tensor(rows), :n].cpu().numpy()
    want_cs = oracle.gemm_i32(np.ascontiguousarray(ra_h).reshape(-1), rb_all.reshape(-1), S, len(rows), n,
                              n).reshape(S, len(rows), n)
    assert np.array_equal(cs_rows, want_cs)
    # FP64 on the sampled rows: exact CRT bit for bit, the reference's reconstruction within tolerance
    c_rows = C.view(n, n)[torch.as_tensor(rows)].cpu().numpy()
    cx = oracle.recon(np.ascontiguousarray(cs_rows).reshape(-1), len(rows), n, dA_h[rows], dB_h, op,
                      exact=True).reshape(len(rows), n)
    assert np.array_equal(c_rows.view(np.uint64), cx.view(np.uint64))
    cf = oracle.recon(np.ascontiguousarray(cs_rows).reshape(-1), len(rows), n, dA_h[rows], dB_h, op,
                      exact=False).reshape(len(rows), n)
    bound = _tolerance(op, plan, dA_h[rows], dB_h, 2) + 2 * np.spacing(np.abs(cf))
    assert np.all(np.abs(c_rows - cf) <= bound)
    e_b200, e_ref = oracle.maxrel_f128_rows(a, b, [c_rows, cf], n, n, n, rows)
    assert e_b200 <= 2 * e_ref, (e_b200, e_ref)
    # the public API gives the same C
    del ra, rb, cs
    ctx_c = np.empty(n * n)
    info = oztt.Context().gemm(a, b, ctx_c, n, n, n, oztt.Options(format=oztt.Format.INT8,
                                                                 reconstruction=oztt.Reconstruction.TwoPass))
    assert info.reconstruction_passes == 2 and info.moduli == case["S"]
    assert np.array_equal(ctx_c.view(np.uint64), C.cpu().numpy().view(np.uint64))
