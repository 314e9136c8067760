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
