"""Shared test set-up: import paths, the `gpu` marker and common fixtures.

`-m "not gpu"` runs on a CPU-only machine (oracle vs golden vectors, host
logic, ABI loading); `-m gpu` runs the CUDA parity tests on a B200.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "cascade-llm_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for path in (REPO, PKG):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: regenerates the full 8B seeded model on the CPU")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA GPU (run the gpu tests on a B200)")
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def golden_path(name):
    return os.path.join(GOLDEN, name)
