"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs everywhere (oracle, host logic, C-ABI load checks);
`-m gpu` needs an sm_100 device and calls the CUDA kernels through the C ABI.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def port():
    import oracle
    return oracle.port()


@pytest.fixture(scope="session")
def ctx():
    from qwen382743090_b200 import build, runtime
    build.build()
    c = runtime.Context(0)
    yield c
    c.close()
