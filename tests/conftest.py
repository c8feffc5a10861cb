"""Shared pytest configuration.

Markers: ``gpu`` — needs a CUDA device (B200); everything else runs on CPU.
The product package lives in a directory whose name is not a Python
identifier, so its directory is put on sys.path and the package is imported
as ``engine``; the checker is imported as ``oracle.oracle``.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "aima-intel-plk-qwen36-35b-u4-engine_b200"
for p in (str(ROOT), str(PKG_DIR), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _no_device_wait_timeouts(request):
    """Every GPU test also fails if a bounded device wait gave up during it."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from engine import _native
    torch.cuda.synchronize()
    n = _native.wait_timeouts(reset=True)
    assert n == 0, f"{n} bounded device waits gave up during this test"
