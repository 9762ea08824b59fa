"""The CTA-pair variant of the residue GEMM (tcgen05.mma.cta_group::2, selected with
oztt_set_option(OZTT_OPT_GEMM_CTA_PAIRS, 1)) against torch's int8 matmul and the oracle, including row
counts that leave the last pair tile half empty (mp an odd multiple of 128); and the integer-pipe
reconstruction (OZTT_OPT_RECON_INT) against the oracle."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture()
def pairs(oztt):
    old = oztt.get_option(oztt.OPT_GEMM_CTA_PAIRS)
    oztt.set_option(oztt.OPT_GEMM_CTA_PAIRS, 1)
    yield
    oztt.set_option(oztt.OPT_GEMM_CTA_PAIRS, old)


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("mp,np_,kp,bfix", [(128, 256, 128, 54), (384, 512, 384, 56), (1280, 768, 2048, 61)])
def test_pair_residue_gemm_mode0(oztt, oracle, cuda, pairs, mp, np_, kp, bfix):
    a, b = oracle.gen_inputs(mp, np_, kp, 0.5, 3)
    plan = oztt.ii_int8_plan(a, b, mp, np_, kp, fixed_bits=bfix, reconstruction=1, max_moduli=24)
    S = plan.S
    g = torch.Generator().manual_seed(mp + np_)
    A = torch.randint(-127, 128, (S, mp, kp), dtype=torch.int8, generator=g).cuda()
    B = torch.randint(-127, 128, (S, np_, kp), dtype=torch.int8, generator=g).cuda()
    out = torch.full((S, mp, np_), 7, dtype=torch.int32, device="cuda")
    oztt.call("oztt_ii_residue_gemm", A.data_ptr(), B.data_ptr(), mp, np_, kp, plan, 0, out.data_ptr(), _stream())
    torch.cuda.synchronize()
    for s in range(S):
        assert torch.equal(out[s], torch._int_mm(A[s], B[s].t())), s


def test_pair_pipeline_and_diagonals(oztt, oracle, cuda, pairs):
    m, n, k = 300, 200, 500
    a, b = oracle.gen_inputs(m, n, k, 0.5, 8)
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    c = oztt.ii_int8_run(a, b, m, n, k, plan)
    rc, ref, _, _ = oracle.emulate(a, b, m, n, k, exact=True)
    assert rc == 0 and np.array_equal(c.view(np.uint64), ref.view(np.uint64))
    iplan = oztt.i_int8_plan(a, b, m, n, k, slices=7)
    ci = oztt.i_int8_run(a, b, m, n, k, iplan)
    refi = oracle.i_emulate(a, b, m, n, k, 7, exact=True)
    assert np.array_equal(ci.view(np.uint64), refi.view(np.uint64))


def test_integer_pipe_reconstruction(oztt, oracle, cuda):
    m, n, k = 260, 300, 400
    a, b = oracle.gen_inputs(m, n, k, 1.0, 12)
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    rc, ref, _, _ = oracle.emulate(a, b, m, n, k, exact=True)
    assert rc == 0
    old = oztt.get_option(oztt.OPT_RECON_INT)
    oztt.set_option(oztt.OPT_RECON_INT, 1)
    try:
        c = oztt.ii_int8_run(a, b, m, n, k, plan)
    finally:
        oztt.set_option(oztt.OPT_RECON_INT, old)
    assert np.array_equal(c.view(np.uint64), ref.view(np.uint64))
