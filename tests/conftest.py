"""Shared test setup.

Markers: ``gpu`` tests need a B200 and the built libdsv4cu.so; everything else
runs on the CPU. The CPU checkers (oracle/) are test infrastructure only.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "deepseek-v4-in-c_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libdsv4cu.so")


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.RefLib.available():
        pytest.skip("reference library oracle/_ref/libdsv4ref.so not built")
    return oracle.RefLib()


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def dev():
    if not _has_gpu():
        pytest.fail("gpu test selected but no CUDA device is visible")
    import dsv4cu
    d = dsv4cu.Device(0)
    yield d
    d.check_status()
    d.close()


@pytest.fixture(autouse=True)
def _device_status(request):
    """After every GPU test: no kernel may have hit a bounded-wait timeout."""
    yield
    if "dev" in request.fixturenames:
        request.getfixturevalue("dev").check_status()


@pytest.fixture(scope="session")
def host():
    if not _has_gpu():
        pytest.fail("gpu test selected but no CUDA device is visible")
    import dsv4cu
    return dsv4cu.HostAPI()


def golden(name: str):
    import numpy as np
    path = os.path.join(GOLDEN, name)
    return np.load(path, allow_pickle=False)
