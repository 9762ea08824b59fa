"""The Scheme II plan made from statistics measured on the device (oztt_ii_int8_plan_device, the path
of Context::gemm) against the host planner, which matches the reference's planner bit for bit: every
field of the plan, the five input statistics included, must be identical."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


CASES = [("uniform", 128, 128, 128, -1.0, {}), ("phi0.5", 300, 200, 500, 0.5, {}), ("phi4", 97, 131, 77, 4.0, {}),
         ("ragged", 1, 70, 1000, 1.0, {}), ("two-pass", 256, 256, 256, 2.0, {"reconstruction": 2}),
         ("max16", 200, 100, 300, 0.5, {"max_moduli": 16}), ("fixed-auto", 64, 64, 64, 1.0, {"fixed_bits": 58}),
         ("tiny-a", 150, 90, 260, 1.0, {}), ("tiny-b", 70, 180, 333, 1.0, {}), ("near-bound", 129, 65, 200, 1.0, {}),
         ("large-scale", 100, 100, 100, 1.0, {})]


@pytest.mark.parametrize("name,m,n,k,phi,kw", CASES)
def test_device_plan_equals_host_plan(oztt, oracle, cuda, name, m, n, k, phi, kw):
    a, b = oracle.gen_inputs(m, n, k, phi, 21)
    if name == "ragged":
        a[: k // 3] = 0.0  # a run of zeros and a row scale far from the others
        b[::7] *= 2.0 ** -40
    # Nonzero magnitudes below 2^-383 send the device statistics to their scale-first recomputation;
    # at and above it the unscaled sums, scaled afterwards, must give the same bits.
    if name == "tiny-a":
        a[5], a[17], a[k + 3] = 2.0 ** -500, 5e-324, -(2.0 ** -384)
    if name == "tiny-b":
        b[3], b[n + 1] = -(2.0 ** -700), 2.0 ** -1000
    if name == "near-bound":
        a[::11] = 2.0 ** -383
        b[::13] = -(2.0 ** -383)
    if name == "large-scale":
        a *= 2.0 ** 100
        b *= 2.0 ** -100
        a[::9] = 2.0 ** -280
        b[::5] = 2.0 ** -380
    host = oztt.ii_int8_plan(a, b, m, n, k, **kw)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dev = oztt.ii_int8_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, stream=_stream(), **kw)
    for f in ("TA", "TB", "nA", "nB", "nC", "recon1_log2"):
        assert np.float64(getattr(dev, f)).view(np.uint64) == np.float64(getattr(host, f)).view(np.uint64), (name, f)
    assert bytes(dev) == bytes(host), name


def test_context_uses_the_same_plan(oztt, oracle, cuda):
    m, n, k = 333, 222, 444
    a, b = oracle.gen_inputs(m, n, k, 0.5, 5)
    opts = oztt.Options(format=oztt.Format.INT8)
    c = np.empty(m * n)
    info = oztt.Context().gemm(a, b, c, m, n, k, opts)
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    assert (info.moduli, info.integer_bits, info.reconstruction_passes) == (plan.S, plan.b, 2 if plan.two_pass else 1)
    ref = oztt.ii_int8_run(a, b, m, n, k, plan)
    assert np.array_equal(c.view(np.uint64), ref.view(np.uint64))


def test_tiled_plan_on_one_rank_equals_host_plan(oztt, oracle, cuda):
    """The tiled statistics (panel measurements, the sketch chain, the host combination) on a 1 x 1 grid,
    without torch.distributed: the plan of the host planner, byte for byte."""
    from oztt_b200.distributed import DeviceStats, Grid, GridComm, plan_ii_int8_tiled

    for (m, n, k, phi) in [(200, 300, 160, 1.0), (77, 65, 513, 4.0)]:
        a, b = oracle.gen_inputs(m, n, k, phi, 13)
        A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        plan = plan_ii_int8_tiled(GridComm(Grid(1, 1, 0, 0)), A, B, m, n, k, stats=DeviceStats(_stream()))
        assert bytes(plan) == bytes(oztt.ii_int8_plan(a, b, m, n, k))
