"""Shared test set-up: the `gpu` marker, import paths, and small helpers."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for path in (ROOT, os.path.join(ROOT, "oracle")):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    import fa_oracle
    fa_oracle.load()
    return fa_oracle


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for -m gpu tests")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"sm_100 device required, found compute capability {major}.x")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)
