"""C-ABI surface and host-side front end of liboztt.so (CPU only: no kernel is launched).

Ports the host-only part of the reference's tests/correctness.cpp (host_validation, :49-85): invalid
calls are rejected with std::invalid_argument (ValueError here / OZTT_EINVAL in the C ABI) before the
device is used, and C stays untouched.
"""

import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "oztt_cuda.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|void|uint64_t|const char\*)\s+(oztt_[a-z0-9_]+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol(oztt):
    names = declared_symbols()
    assert len(names) >= 12
    for name in names:
        assert hasattr(oztt.lib, name), f"{name} is declared in include/oztt_cuda.h but not exported"
    assert set(names) == set(oztt.C_ABI_SYMBOLS)


def test_cpp_api_symbols_exported(oztt):
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(oztt.library_path)], capture_output=True,
                         text=True).stdout
    for sym in ["_ZN8ozTTgemm12is_availableENS_6FormatE", "_ZN8ozTTgemm11format_nameENS_6FormatE",
                "_ZN8ozTTgemm7ContextC1ENS_13DeviceOptionsE", "_ZN8ozTTgemm7ContextD1Ev"]:
        assert sym in out
    assert "_ZN8ozTTgemm7Context4gemm" in out and "_ZN8ozTTgemm7Context8multiply" in out


def test_epilogue_division_magic(oztt):
    """floor(a/m) as computed by the GEMM epilogue, for every INT8 modulus and a < 2^31."""
    rng = np.random.default_rng(0)
    samples = np.concatenate([np.arange(0, 70000), rng.integers(0, 2**31, 20000),
                              np.array([2**31 - 1, 2**31 - 2, 2**30, 2**24 - 1, 2**24])]).astype(np.uint64)
    f = oztt.lib.oztt_test_udiv_small
    for d in list(range(3, 256)):
        # all multiples near the top of the range plus the samples
        extra = np.array([(2**31 - 1) // d * d, (2**31 - 1) // d * d - 1], dtype=np.uint64)
        for a in np.concatenate([samples[::97], extra]):
            assert f(int(a), d) == int(a) // d, (int(a), d)
    # exhaustive over the 16-bit range used for r*y
    for d in (3, 29, 37, 127, 151, 199, 211, 254, 255):
        a = np.arange(0, 65536)
        got = np.array([f(int(x), d) for x in a[::7]])
        assert np.array_equal(got, a[::7] // d)


def test_is_available_and_names(oztt):
    assert oztt.is_available(oztt.Format.INT8) and oztt.is_available(oztt.Format.FP8)
    for f in (oztt.Format.BFP8, oztt.Format.BFP4, oztt.Format.BFP2):
        assert not oztt.is_available(f)
    assert [oztt.format_name(f) for f in oztt.Format] == ["BF16", "FP16", "TF32", "BFP8", "FP8", "INT8", "BFP4",
                                                          "BFP2"]
    assert oztt.format_name(100) == "unknown"


def test_host_validation(oztt):
    """tests/correctness.cpp:49-85 of the reference, through the C ABI (oztt_gemm)."""
    ctx = oztt.Context()
    a = np.ones(4)
    b = np.ones(4)
    c = np.full(4, 123.0)
    opt = oztt.Options(format=oztt.Format.INT8)

    def invalid(**kw):
        args = dict(a=a, b=b, c=c, m=2, n=2, k=2, options=opt)
        args.update(kw)
        with pytest.raises(ValueError):
            ctx.gemm(args["a"], args["b"], args["c"], args["m"], args["n"], args["k"], args["options"])

    invalid(m=0)
    invalid(n=3)
    invalid(options=oztt.Options(scheme=100, format=oztt.Format.INT8))
    invalid(options=oztt.Options(format=100))
    invalid(options=oztt.Options(format=oztt.Format.INT8, slices=10))
    invalid(options=oztt.Options(scheme=oztt.Scheme.I, format=oztt.Format.INT8,
                                 reconstruction=oztt.Reconstruction.TwoPass))
    invalid(options=oztt.Options(format=oztt.Format.INT8, max_moduli=25))
    invalid(options=oztt.Options(scheme=oztt.Scheme.I, format=oztt.Format.INT8, slices=257))
    invalid(options=oztt.Options())  # default format BFP8 is not available on B200
    a2 = a.copy()
    a2[0] = np.nan
    invalid(a=a2)
    b2 = b.copy()
    b2[0] = np.inf
    invalid(b=b2)
    invalid(a=np.full(4, 2.0 ** -130))
    invalid(a=np.full(4, 2.0 ** 128))
    assert np.all(c == 123.0), "invalid input modified the output"


def test_context_rejects_negative_device(oztt):
    with pytest.raises(ValueError):
        oztt.Context(oztt.DeviceOptions(device_id=-1))


def test_plan_rejections(oztt):
    """Two moduli cannot cover an FP64-equivalent width (reference tests/correctness.cpp:297-306):
    std::runtime_error, before any device work."""
    a = np.ones(64 * 64)
    with pytest.raises(RuntimeError, match="max_moduli"):
        oztt.ii_int8_plan(a, a, 64, 64, 64, max_moduli=2)
    with pytest.raises(ValueError):
        oztt.ii_int8_plan(a, a, 64, 64, 64, max_moduli=25)
    # K so large that the INT8 moduli shrink below the window even with 24 moduli
    k = 1 << 24
    with pytest.raises(RuntimeError, match="K="):
        oztt.ii_int8_plan(np.ones(k), np.ones(k), 1, 1, k, fixed_bits=0, reconstruction=1)


def test_eval_generator_matches_oracle(oztt, oracle):
    """The library's evaluation generator and hash equal the oracle's restatement (which reproduces the
    reference's published hash from the same inputs)."""
    for (m, n, k, phi, seed) in [(5, 7, 3, -1.0, 7), (16, 8, 4, 0.5, 0), (3, 3, 3, 4.0, 123)]:
        a1, b1 = oztt.eval_inputs(m, n, k, phi, seed)
        a2, b2 = oracle.gen_inputs(m, n, k, phi, seed)
        assert np.array_equal(a1, a2) and np.array_equal(b1, b2)
        assert oztt.eval_output_hash(a1) == oracle.output_hash(a2)
