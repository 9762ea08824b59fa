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
