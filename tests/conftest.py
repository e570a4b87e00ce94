"""Shared pytest setup: the `gpu` marker, repo-root imports, oracle build."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def cuda_device():
    """The CUDA device for GPU tests. Fails (does not skip) without a GPU, so a
    GPU run can never pass silently on a host fallback."""
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"kernels target sm_100a, found sm_{major}{minor}"
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(autouse=True)
def _check_device_error_word(request):
    """After every GPU test, the kernels' device error word must be clear."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from lema_b200 import _native
    assert _native.device_error() == 0, "a kernel recorded a device-side failure"
