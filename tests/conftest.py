"""Shared pytest configuration. GPU tests carry @pytest.mark.gpu and run only
with `-m gpu` on a B200; everything else runs on CPU."""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100a device (B200)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import bridge

    bridge.lib()
    return bridge


@pytest.fixture(scope="session")
def rns8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200
