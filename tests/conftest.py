import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "sglang-mlx_b200"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); calls libkvcache kernels")


@pytest.fixture(scope="session")
def gpu():
    """The CUDA path, required (never skipped): a GPU test without a device fails."""
    from sglang_mlx_b200 import _lib

    n = _lib.device_count()
    if n < 1:
        pytest.fail("no CUDA device visible to libkvcache")
    _lib.set_device(0)
    _lib.get_status(0, clear=True)
    return _lib


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden.npz")))
