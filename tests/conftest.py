"""Shared test setup: import paths, the `gpu` marker, seeded fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "static-lm_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    """torch with a visible CUDA device; GPU tests fail (not skip) without one."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    torch.cuda.init()
    return torch
