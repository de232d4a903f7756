"""Test configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs the oracle against the golden vectors, the host logic
and the C-ABI library's load/export checks, with no GPU.  ``-m gpu`` runs the
parity tests proper: every CUDA path through the C ABI against the oracle.
"""
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (parity tests through the C ABI)")
    config.addinivalue_line("markers", "slow: long-running")


def golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def gpu():
    """The B200 target; the GPU tests fail (not skip) when it cannot run."""
    import torch
    from superfloat.python_b200 import build, _lib
    from superfloat.python_b200._device import get_device
    build.build()
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    _lib.ensure_device(0)
    return get_device("b200")


@pytest.fixture
def rng():
    return np.random.default_rng(int(os.environ.get("SF_TEST_SEED", "0")))
