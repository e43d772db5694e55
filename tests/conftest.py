import os
import sys

import pytest

# One hardware work queue per persistent kernel: keep other streams off it (see
# gpuos_b200/__init__.py); must be set before CUDA initialises.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def rt():
    """The gpuos_ext module with a runtime initialised on cuda:0 for the whole session."""
    import torch
    from gpuos_b200 import gpuos_ext
    torch.cuda.init()
    gpuos_ext.init(capacity=8192, threads_per_block=256)
    yield gpuos_ext
    gpuos_ext.shutdown()
