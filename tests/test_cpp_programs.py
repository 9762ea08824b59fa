"""The C++ programs built against the public API (include/ozTTgemm/ozTTgemm.hpp)."""

import subprocess
from pathlib import Path

import pytest

BUILD = Path(__file__).resolve().parent.parent / "oztt_b200" / "_build"


def run(name, *args):
    exe = BUILD / name
    assert exe.exists(), f"{exe} is not built (python -m oztt_b200.build)"
    return subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=600)


def test_correctness_host_only():
    r = run("correctness", "--host-only")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "input validation passed" in r.stdout


@pytest.mark.gpu
def test_correctness_program():
    r = run("correctness")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all correctness checks passed" in r.stdout


@pytest.mark.gpu
def test_gemm_example():
    r = run("gemm_example")
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.split() == ["58", "64", "139", "154"]


# ---- the reference's own callers, compiled unchanged against this library (oracle/Makefile, callers) ----
REF_BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref"
QUICK = Path(__file__).resolve().parent / "golden" / "quick_table_128.json"


def run_ref(name, *args, cwd=None):
    exe = REF_BIN / name
    if not exe.exists():
        pytest.skip(f"{exe} is not built (make -C oracle callers, in the build container)")
    return subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=900, cwd=cwd)


def test_reference_correctness_host_only():
    """The reference's tests/correctness.cpp --host-only: its input-validation cases against this library."""
    r = run_ref("ref_correctness", "--host-only")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "input validation passed" in r.stdout


def test_reference_evaluator_lists_the_table():
    r = run_ref("ref_evaluate", "--suite", "table", "--quick", "--formats", "BF16,FP16,TF32,FP8,INT8", "--list")
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.strip().splitlines()
    assert lines[0].startswith("suite,n,scheme,format") and len(lines) == 11


@pytest.mark.gpu
def test_reference_correctness_program():
    """The reference's whole acceptance test: every format and scheme against long double, the overlap and
    rejection cases, and its checks of the evaluator hooks (phase timing, whole-pass replay, fixed width)."""
    r = run_ref("ref_correctness")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all correctness checks passed" in r.stdout


@pytest.mark.gpu
def test_reference_gemm_example():
    r = run_ref("ref_gemm_example")
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.split() == ["58", "64", "139", "154"]


@pytest.mark.gpu
def test_reference_evaluator_quick_table(oztt, oracle, tmp_path):
    """The reference's evaluator (evaluation/evaluate.cpp, unchanged) in its quick table mode on B200, with
    its phase timing and whole-pass replay checks. Every row's plan (slices, width, moduli, passes, partial
    products) equals the reference device's published run (tools/validated/quick.csv) and its accuracy
    matches to 1e-3; the output is the B200 pipeline's exact reconstruction, so its hash is that of the
    oracle's exact restatement (the reference device's own reconstruction rounds differently in the last
    bits; the published hashes are reproduced from the B200 products in test_gpu_digit, test_gpu_scheme1
    and test_gpu_ii_int8)."""
    import csv
    import json

    out = tmp_path / "quick.csv"
    r = run_ref("ref_evaluate", "--suite", "table", "--quick", "--formats", "BF16,FP16,TF32,FP8,INT8", "--output",
                str(out))
    assert r.returncode == 0, r.stdout + r.stderr
    with out.open() as f:
        got = {(row["scheme"], row["format"]): row for row in csv.DictReader(f)}
    want = json.loads(QUICK.read_text())["rows"]
    assert len(got) == len(want) == 10
    n = 128
    a, b = oracle.gen_inputs(n, n, n, -1.0, 7)
    for w in want:
        g = got[(w["scheme"], w["format"])]
        for key in ("slices", "integer_bits", "moduli", "passes", "partial_products"):
            assert g[key] == w[key], (w["scheme"], w["format"], key, g[key], w[key])
        rel, want_rel = float(g["relative_fro"]), float(w["relative_fro"])
        assert abs(rel - want_rel) <= 1e-3 * want_rel, (w["scheme"], w["format"], rel, want_rel)
        fmt = int(oztt.Format[w["format"]])
        if w["scheme"] == "I":
            exact = oracle.i_emulate(a, b, n, n, n, int(w["slices"]), exact=True, fmt=fmt)
        elif w["format"] == "INT8":
            rc, exact, _, err = oracle.emulate(a, b, n, n, n, max_moduli=16, passes=1, fixed_bits=54, exact=True)
            assert rc == 0, err
        else:
            max_moduli = {"BF16": 24, "FP16": 24, "TF32": 11, "FP8": 14}[w["format"]]
            fp = oztt.digit_plan(a, b, n, n, n, max_moduli=max_moduli, reconstruction=1, fixed_bits=54, fmt=fmt)
            rc, exact, err = oracle.digit_emulate(a, b, n, n, n, fp, exact=True)
            assert rc == 0, err
        assert int(g["output_hash"], 16) == int(oracle.output_hash(exact), 16), (w["scheme"], w["format"])
        assert float(g["total_ms"]) > 0 and float(g["effective_tflops"]) > 0
