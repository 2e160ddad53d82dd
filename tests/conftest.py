import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "asdsl-framework_b200")
for p in (PKG_DIR, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running (full-size shapes)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build

    build()
    return Oracle()


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))

    return load


@pytest.fixture(scope="session")
def native():
    """The CUDA library, built in-tree if needed; GPU tests fail loudly without it."""
    from asdsl_b200 import _lib
    from asdsl_b200.build import build_library

    build_library()
    _lib.load()
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is available")
    return _lib
