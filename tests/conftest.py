"""Shared pytest setup: markers, import paths, common fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fp4-gemm-blackwell_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"needs sm_100 (B200), found sm_{major}{minor}"
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def fp4():
    """The drop-in fp4_gemm module (loads libfp4gemm.so; never an oracle)."""
    import fp4_gemm
    return fp4_gemm
