"""pytest configuration: the `gpu` marker and the shared fixtures.

`-m "not gpu"` runs on any machine: the oracle against the reference's published golden values and
against the reference's own host code compiled in place, the planner, the C-ABI surface and the
front-end validation (all host code). `-m gpu` runs the CUDA kernels on a B200 through the C ABI
and compares them with the oracle.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle_lib import Oracle, RefEmu, RefPlan, RefPlan1, RefPlanDigit  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def oracle():
    return Oracle()


@pytest.fixture(scope="session")
def ref_plan():
    try:
        return RefPlan()
    except FileNotFoundError:
        pytest.skip("oracle/_ref was not built on this machine (needs the reference tree)")


@pytest.fixture(scope="session")
def ref_plan1():
    try:
        return RefPlan1()
    except FileNotFoundError:
        pytest.skip("oracle/_ref was not built on this machine (needs the reference tree)")


@pytest.fixture(scope="session")
def ref_plan1_r64():
    try:
        return RefPlan1(r64=True)
    except FileNotFoundError:
        pytest.skip("oracle/_ref was not built on this machine (needs the reference tree)")


@pytest.fixture(scope="session")
def ref_plan1_f8():
    try:
        return RefPlan1(fp8=True)
    except FileNotFoundError:
        pytest.skip("oracle/_ref was not built on this machine (needs the reference tree)")


@pytest.fixture(scope="session")
def ref_plan_digit():
    """ref_plan_digit(fmt): the reference's planner compiled for that digit format (skips without it)."""
    cache = {}

    def get(fmt):
        if fmt not in cache:
            try:
                cache[fmt] = RefPlanDigit(fmt)
            except FileNotFoundError:
                pytest.skip("oracle/_ref was not built on this machine (needs the reference tree)")
        return cache[fmt]

    return get


@pytest.fixture(scope="session")
def ref_plan_f8():
    try:
        return RefPlanDigit(4)
    except FileNotFoundError:
        pytest.skip("oracle/_ref was not built on this machine (needs the reference tree)")


@pytest.fixture(scope="session")
def ref_emu():
    try:
        return RefEmu()
    except FileNotFoundError:
        pytest.skip("oracle/_ref was not built on this machine (needs the reference tree)")


@pytest.fixture(scope="session")
def oztt():
    import oztt_b200

    return oztt_b200


@pytest.fixture(scope="session")
def cuda():
    """The torch CUDA device for GPU tests; a GPU test on a machine without one fails loudly."""
    import torch

    assert torch.cuda.is_available(), "this test needs a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"expected a B200 (sm_100), found sm_{major}{minor}"
    return torch.device("cuda:0")
