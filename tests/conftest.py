"""Shared fixtures. GPU tests carry @pytest.mark.gpu and call the CUDA
library through its C ABI; everything else runs on a CPU-only machine."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    config.addinivalue_line("markers", "slow: full-size parity (seconds of oracle work)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, have_reference
    if not have_reference():
        pytest.skip("reference build oracle/_ref not present")
    return Reference()


@pytest.fixture(scope="session")
def sicu():
    """The CUDA library, initialised on device 0 (GPU tests only)."""
    import torch
    from siphon_b200 import lib
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    torch.cuda.init()
    s = lib.load()
    s.init(0)
    return s


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"
