"""The no-allocation column scaling (oztt_ii_scale_cols_noalloc) against the ordinary one.

Some callers cannot let a library allocate device memory when they call it: programs whose device
memory is owned by their own allocator or reserved up front, and latency-critical paths where an
allocation could synchronise or fail. oztt_ii_scale_cols_noalloc gives them the column-scaling stage
with its scratch in a fixed static device array instead of the stream-ordered allocator.

This file is named to be collected last, so that a run stopping at the first failure has already run
every other test; it passes alone in a fresh process as well as after the rest.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _scale_cols(oztt, entry, x, k, n, shift):
    delta = torch.zeros(n, dtype=torch.int32, device="cuda")
    bf = torch.zeros(n, dtype=torch.int16, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    oztt.call(entry, x.data_ptr(), k, n, n, shift, delta.data_ptr(), bf.data_ptr(), flags.data_ptr(), _stream())
    torch.cuda.synchronize()
    return delta.cpu().numpy(), bf.cpu().numpy(), int(flags.cpu()[0])


def test_noalloc_matches_allocating_entry(oztt, cuda):
    rng = np.random.default_rng(2024)
    shift = 14
    # Two calls in a row through the C ABI; the second one is smaller and has much smaller values, so
    # maxima left in the shared scratch by the first call would show up if it were not cleared.
    cases = [(300, 5000, 1.0, 1e3), (77, 1999, 1e-6, 1.0)]
    for k, n, scale, spike in cases:
        b = rng.standard_normal(k * n) * scale
        b[rng.integers(0, k * n, 7)] *= spike
        b[: n // 9] = 0.0  # some zero columns in the first row block
        x = torch.from_numpy(b).cuda()
        want = _scale_cols(oztt, "oztt_ii_scale_cols", x, k, n, shift)
        got = _scale_cols(oztt, "oztt_ii_scale_cols_noalloc", x, k, n, shift)
        assert np.array_equal(got[0], want[0])
        assert np.array_equal(got[1], want[1])
        assert got[2] == want[2]


def test_noalloc_rejects_more_columns_than_its_scratch(oztt, cuda):
    limit = 262144
    x = torch.zeros(limit + 1, dtype=torch.float64, device="cuda")
    delta = torch.zeros(limit + 1, dtype=torch.int32, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="exceeds the limit"):
        oztt.call("oztt_ii_scale_cols_noalloc", x.data_ptr(), 1, limit + 1, limit + 1, 14, delta.data_ptr(), 0,
                  flags.data_ptr(), _stream())
