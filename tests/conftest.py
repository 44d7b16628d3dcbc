import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _no_device_error(request):
    """Every GPU test ends with the engine's device error word clear."""
    yield
    if "gpu" in request.keywords:
        import torch

        if torch.cuda.is_available():
            from spikestack_lite_b200 import _lib

            bits = _lib.device_error(clear=True)
            assert bits == 0, f"engine kernels reported device error bits {bits:#x}"


@pytest.fixture(scope="session")
def ref_engine():
    """The reference's own CUDA engines built from its sources into oracle/_ref
    (oracle/build_ref.py); the test is skipped when they were not built."""
    from oracle.build_ref import load_ref

    def get(name):
        mod = load_ref(name)
        if mod is None:
            pytest.skip(f"reference engine {name} not built (oracle/build_ref.py)")
        return mod

    return get


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = np.load(os.path.join(GOLDEN, name + ".npz"))
        return cache[name]

    return load
