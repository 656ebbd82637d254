"""Shared pytest setup: the `gpu` marker, import paths and small helpers.

`-m "not gpu"` runs on any machine (oracle, host logic, C-ABI loading and
argument validation, CPU gloo ranks). `-m gpu` needs a B200 and calls the
CUDA library through its C ABI.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "flash-attention-v4-rocm_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def lib():
    import fav4_bshd
    return fav4_bshd.load_library()


@pytest.fixture(scope="session")
def runner(lib):
    import fav4_bshd
    return fav4_bshd.Runner(lib)


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"sm_100 required, found sm_{major}{minor}"
    return torch.device("cuda:0")
