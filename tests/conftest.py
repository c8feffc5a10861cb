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


@pytest.fixture(scope="session")
def config1():
    """BASELINE config 1 weights: 256 experts (gate_up [1024, 2048], down
    [2048, 512], u4 g128), one shared expert, fp16 router and shared gate."""
    import numpy as np
    from helpers import make_bank
    rng = np.random.default_rng(101)
    h, i, e = 2048, 512, 256
    bank = make_bank(rng, e, h, i)
    shared = make_bank(rng, 1, h, i)
    w_router = (rng.standard_normal((e, h)) * 0.02).astype(np.float16)
    w_sg = (rng.standard_normal((1, h)) * 0.02).astype(np.float16)
    x = rng.standard_normal(h).astype(np.float16)
    return dict(bank=bank, shared=shared, w_router=w_router, w_sg=w_sg, x=x)
