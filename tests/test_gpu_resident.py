"""Resident operands (oztt_resident_*): products of matrices kept in HBM equal Context::gemm's, bit for bit,
with the same Info, whatever the operands were multiplied with before (cached measurements and residue
planes); host or device inputs and outputs; the front end's value checks at creation."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _context(oztt, a, b, m, n, k, **kw):
    c = np.empty(m * n)
    info = oztt.Context().gemm(a, b, c, m, n, k, oztt.Options(format=oztt.Format.INT8, **kw))
    return c, info


@pytest.mark.parametrize("m,n,k,phi", [(300, 200, 500, 1.0), (1000, 700, 1100, 0.5), (65, 129, 33, 4.0)])
def test_resident_products_equal_context(oztt, oracle, cuda, m, n, k, phi):
    a, b = oracle.gen_inputs(m, n, k, phi, 3)
    a2, _ = oracle.gen_inputs(m, 1, k, phi + 0.5, 4)
    RA, RA2 = oztt.ResidentMatrix(a, m, k, "A"), oztt.ResidentMatrix(a2, m, k, "A")
    RB = oztt.ResidentMatrix(torch.from_numpy(b).cuda(), k, n, "B")  # from device memory
    for (ra, av) in ((RA, a), (RA2, a2), (RA, a)):  # B's planes are reused across the three products
        c, info = oztt.resident_gemm(ra, RB)
        want, winfo = _context(oztt, av, b, m, n, k)
        assert np.array_equal(c.view(np.uint64), want.view(np.uint64))
        assert info == winfo
    # options, and C in device memory
    for kw in ({"reconstruction": oztt.Reconstruction.TwoPass}, {"max_moduli": 18}):
        cd = torch.empty(m * n, dtype=torch.float64, device="cuda")
        _, info = oztt.resident_gemm(RA, RB, cd, oztt.Options(format=oztt.Format.INT8, **kw))
        want, winfo = _context(oztt, a, b, m, n, k, **kw)
        assert np.array_equal(cd.cpu().numpy().view(np.uint64), want.view(np.uint64))
        assert info == winfo
    for r in (RA, RA2, RB):
        r.close()


def test_resident_checks(oztt, oracle, cuda):
    a, b = oracle.gen_inputs(20, 30, 40, 1.0, 9)
    bad = a.copy()
    bad[7] = np.nan
    with pytest.raises(ValueError, match="A contains NaN or infinity"):
        oztt.ResidentMatrix(bad, 20, 40, "A")
    tiny = b.copy()
    tiny[:] = 2.0 ** -130
    with pytest.raises(ValueError, match="must be in"):
        oztt.ResidentMatrix(tiny, 40, 30, "B")
    RA, RB = oztt.ResidentMatrix(a, 20, 40, "A"), oztt.ResidentMatrix(b, 40, 30, "B")
    with pytest.raises(ValueError, match="left"):
        oztt.resident_gemm(RB, RA)
    with pytest.raises(ValueError, match="INT8"):
        oztt.resident_gemm(RA, RB, options=oztt.Options(format=oztt.Format.FP8))
    RC = oztt.ResidentMatrix(b, 40, 30, "A")
    with pytest.raises(ValueError, match="span sizes"):
        oztt.resident_gemm(RA, oztt.ResidentMatrix(a, 20, 40, "B"))
    RC.close()
