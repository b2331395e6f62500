"""Shared pytest set-up: import paths and the `gpu` marker.

`-m "not gpu"` runs the oracle, host-logic and library-loading tests on any
machine; `-m gpu` runs the parity tests through the C ABI on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("flash-attention-cpu_b200", "oracle", "tests"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def gpu_lib():
    """The product library, with a GPU present (the test is skipped elsewhere)."""
    import fa_b200
    if fa_b200.device_count() == 0:
        pytest.skip("no CUDA device")
    return fa_b200
