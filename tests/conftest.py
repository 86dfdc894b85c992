"""Shared test set-up: import paths, the `gpu` marker, and the built library.

`-m "not gpu"` runs on a host without a GPU (oracle, golden vectors, host logic,
C-ABI exports, gloo ranks); `-m gpu` runs the parity tests on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flash-attention-p100_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


def pytest_sessionstart(session):
    # Build the library up front (no-op when it is current) so a missing nvcc
    # or a compile error shows up once, not as a failure in every test.
    import _build
    _build.build()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"needs an sm_100 device, found sm_{major}x")
    return torch.device("cuda", 0)
