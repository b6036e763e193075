"""Shared test setup: registers the ``gpu`` marker, puts the repository root on sys.path
and builds the CPU oracle (test infrastructure) before any test uses it."""
from __future__ import annotations

import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return {k["name"]: k for k in json.load(f)["kats"]}


@pytest.fixture(scope="session")
def fixtures():
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, "oracle_fixtures.npz")))


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import rustllm_b200
    rustllm_b200.load()
    return torch.device("cuda", 0)
