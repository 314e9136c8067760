import json
import os
import sys

import pytest

TESTS = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(TESTS)
for p in (TESTS, os.path.join(REPO, "oracle"), os.path.join(REPO, "project-zero_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    with open(os.path.join(TESTS, "golden", "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build(ref=False)
    return oracle.Oracle()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="session")
def pz(cuda):
    import pz_sampling
    return pz_sampling


@pytest.fixture(scope="session")
def pz_cpu():
    """The library's host-only entry points (no kernel is launched)."""
    import pz_sampling
    return pz_sampling


def pytest_terminal_summary(terminalreporter):
    """Reports the boundary cases (draws within 1e-6 of a CDF edge that gave
    a different id than the oracle) counted by the parity tests."""
    try:
        from gpu_helpers import BOUNDARY_LOG
    except ImportError:
        return
    if not BOUNDARY_LOG:
        return
    rows = sum(n for _, n, _ in BOUNDARY_LOG)
    cases = sum(c for _, _, c in BOUNDARY_LOG)
    terminalreporter.write_line(f"parity: {cases} boundary case(s) in {rows} sampled rows "
                                f"({len(BOUNDARY_LOG)} comparisons)")
    for label, n, c in BOUNDARY_LOG:
        if c:
            terminalreporter.write_line(f"  {label or '?'}: {c} of {n} rows")
