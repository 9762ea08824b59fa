"""The bounded row statistics of A (band_certify_kernel, oztt_b200/csrc/stats.cu) against numpy.

Each row of the output holds the largest magnitude (as its bit pattern, exact), then sum x^2, the eight
sketch sums sum x y_l, their absolute sums sum |x y_l| and sum |x| ew, all in FP64 in the kernel's order.
The sums are checked against numpy's to a relative 1e-12 of their absolute sums (any order of k terms is
within k u of that), the maxima bit for bit, every row by itself: row counts that end inside a warp's pair
of rows and inside a block of 16 rows, and a column count that ends inside a chunk of the sketch. The
certified plan decision (oztt_b200/csrc/planner.cpp) reads these slots; an earlier form of the kernel put
sum |x| ew into the next row's maximum.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

W = 19


def _numpy_rows(a, y, ew):
    t = a[:, None, :] * y[None, :, :]  # rows x 8 x k
    out = np.zeros((a.shape[0], W))
    out[:, 0] = np.abs(a).max(axis=1)
    out[:, 1] = (a * a).sum(axis=1)
    out[:, 2:10] = t.sum(axis=2)
    out[:, 10:18] = np.abs(t).sum(axis=2)
    if ew is not None:
        out[:, 18] = np.abs(a) @ ew
    return out, np.abs(t).sum(axis=2), (a * a).sum(axis=1)


@pytest.mark.parametrize("rows,k,with_ew", [(37, 700, True), (16, 256, True), (33, 1000, False), (1, 5, True)])
def test_band_certify_rows_match_numpy(oztt, cuda, rows, k, with_ew):
    rng = np.random.default_rng(rows * 1000 + k)
    a = rng.standard_normal((rows, k)) * np.exp2(rng.integers(-20, 20, (rows, 1)))  # rows of other magnitudes
    y = rng.standard_normal((8, k))
    ew = np.abs(rng.standard_normal(k)) * 1e-9 if with_ew else None
    dev = "cuda"
    A = torch.from_numpy(a).to(dev)
    Y = torch.from_numpy(y).to(dev)
    E = torch.from_numpy(ew).to(dev) if with_ew else None
    out = torch.full((rows, W), -7.0, dtype=torch.float64, device=dev)  # every slot must be written
    flags = torch.zeros(4, dtype=torch.int32, device=dev)
    oztt.call("oztt_test_band_certify", A.data_ptr(), rows, k, Y.data_ptr(), E.data_ptr() if with_ew else None,
              out.data_ptr(), flags.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want, abs_sums, s2 = _numpy_rows(a, y, ew)
    # the maxima, bit for bit, in slot 0 of each row (as a magnitude pattern)
    assert np.array_equal(got[:, 0].view(np.uint64), want[:, 0].view(np.uint64))
    # the sums within k u of their absolute sums
    tol = 1e-12
    assert np.all(np.abs(got[:, 1] - want[:, 1]) <= tol * s2)
    assert np.all(np.abs(got[:, 2:10] - want[:, 2:10]) <= tol * abs_sums)
    assert np.all(np.abs(got[:, 10:18] - want[:, 10:18]) <= tol * abs_sums)
    if with_ew:
        assert np.all(np.abs(got[:, 18] - want[:, 18]) <= tol * want[:, 18])
        assert np.all(got[:, 18] > 0)
    else:
        assert np.all(got[:, 18] == 0)
    assert int(flags[0].item()) == 0
