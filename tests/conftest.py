import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session", autouse=True)
def _library_built():
    """The C-ABI tests load mail_b200/libmoe_b200.so; build it (nvcc, no GPU
    needed) when a fresh checkout runs the tests before the build step.
    The library itself never builds on import: a missing library is an
    error there."""
    from mail_b200 import _lib, build

    if not os.path.exists(_lib.LIB_PATH):
        build.build()


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
