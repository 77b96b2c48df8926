"""Shared pytest configuration.

Markers: ``gpu`` tests need a B200 and call the sm_100a kernels through the C
ABI; everything else runs on CPU. GPU tests never skip silently: if CUDA or
the library is missing they fail.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a kernels)")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def oracle():
    from oracle.build_oracle import build_oracle  # noqa: WPS433
    build_oracle()
    import oracle as o  # noqa: WPS433
    return o


@pytest.fixture(scope="session")
def rrlib():
    import raggedroute_b200 as rr  # noqa: WPS433
    rr.lib()
    return rr


@pytest.fixture(scope="session")
def cuda():
    import torch  # noqa: WPS433
    assert torch.cuda.is_available(), "GPU test requested but CUDA is unavailable"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"expected a B200 (sm_100), got sm_{major}{minor}"
    return torch.device("cuda:0")
