"""The bounded waits of the tensor-core GEMM kernels, made to run out on purpose without a fault.

Every mbarrier wait of the residue GEMM gives up after a limit, records an error code and raises an
abort flag that sends the CTA's other roles out of their waits; the host turns the code into a
runtime_error and the CUDA context stays usable. Here a test-only kernel waits, through the GEMM's own
wait routine, on an mbarrier that nothing arrives at (no TMA load or MMA in flight), with a 2 ms limit; a
second thread then waits on the same barrier with the abort flag raised and must leave at once. Then an
ordinary residue GEMM on the same context must still be bit-exact.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def test_gemm_wait_gives_up_and_the_context_stays_usable(oztt, cuda):
    codes = np.zeros(2, dtype=np.int32)
    with pytest.raises(RuntimeError, match="gave up waiting"):
        oztt.call("oztt_test_gemm_wait_timeout", 2_000_000, codes.ctypes.data, _stream())
    assert codes[0] == 8  # ERR_WAIT_EPILOGUE: the code the epilogue's wait records
    assert codes[1] == 1  # the second waiter left on the abort flag
    # the next GEMM on the same context is exact
    a = np.ones(2)
    plan = oztt.ii_int8_plan(a, a, 2, 2, 1, fixed_bits=54, reconstruction=1, max_moduli=16)
    mp, np_, kp = 256, 512, 384
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randint(-127, 128, (plan.S, mp, kp), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-127, 128, (plan.S, np_, kp), dtype=torch.int8, device="cuda", generator=g)
    out = torch.zeros((plan.S, mp, np_), dtype=torch.int32, device="cuda")
    oztt.call("oztt_ii_residue_gemm", A.data_ptr(), B.data_ptr(), mp, np_, kp, plan, 0, out.data_ptr(), _stream())
    torch.cuda.synchronize()
    for s in range(plan.S):
        assert torch.equal(out[s], torch._int_mm(A[s], B[s].t())), s


def test_wait_limit_is_checked(oztt, cuda):
    with pytest.raises(ValueError):
        oztt.call("oztt_test_gemm_wait_timeout", 0, None, _stream())
