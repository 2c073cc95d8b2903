import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and runs libmlkb200 kernels")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name + ".npz"))
    return load


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device (device memory and streams only)."""
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    import mlk2_b200

    assert mlk2_b200.lib().mlkb_device_count() > 0
    return torch


@pytest.fixture(params=["compiled", "interpreted"])
def chain_path(request, cuda):
    """Runs a chain test twice: with chains compiled at run time (NVRTC) and
    on the interpreter kernels; checks through the library's launch counter
    that the compiled kernels really ran in the first case and not in the
    second."""
    from mlk2_b200 import api

    compiled = request.param == "compiled"
    active, _, before = api.chain_compile(1 if compiled else 0)
    assert active == compiled, "NVRTC must be loadable where the GPU tests run"
    try:
        yield request.param
        _, _, after = api.chain_compile(-1)
        assert (after > before) if compiled else (after == before), (request.param, before, after)
    finally:
        api.chain_compile(1)
