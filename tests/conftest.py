"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "oracle"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def oracle():
    from oracle import OracleLib

    return OracleLib()


@pytest.fixture(scope="session")
def cuda_device():
    """The GPU tests never skip: on a box without a device they fail loudly."""
    from mdescriptor_b200.soap import device_count

    count = device_count()
    if count < 1:
        pytest.fail("no CUDA device visible to the mdsoap engine")
    return 0
