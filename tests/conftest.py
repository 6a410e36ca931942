"""Shared pytest setup: import paths, the `gpu` marker, and skips for GPU tests on CPU-only hosts."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "kernel-development_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built libkdb200.so")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def lib():
    from kdb200 import _lib
    return _lib.lib()


@pytest.fixture(autouse=True)
def _clear_device_status(request):
    """GPU tests start and end with a clean device status word; a timeout or bounds report fails the test."""
    if "gpu" not in request.keywords or not _cuda_ok():
        yield
        return
    from kdb200 import _lib
    _lib.status_read(clear=True)
    yield
    st = _lib.status_read(clear=True)
    expected = getattr(request.node, "expected_device_status", 0)
    assert st[0] == expected, f"device status word after test: {st}"
