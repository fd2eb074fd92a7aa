import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the native library")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def sg():
    """The native library through its Python binding (GPU tests)."""
    import torch
    from silicongraph_b200 import _lib, kernels
    if not os.path.exists(_lib.LIB_PATH):
        from silicongraph_b200 import build
        build.build()
    _lib.load()
    torch.cuda.init()
    return kernels


def golden(name):
    import numpy as np
    return np.load(os.path.join(GOLDEN, name))
