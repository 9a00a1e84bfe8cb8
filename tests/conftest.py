"""Test configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on any machine (oracle pins, ABI exports, host logic);
`-m gpu` runs the CUDA parity tests on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_lib():
    from ferry_b200 import build

    build.build()
    from ferry_b200 import _abi

    return _abi.lib()
