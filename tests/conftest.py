"""Shared pytest configuration: the `gpu` marker and common fixtures."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_dev():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _check_device_status(request):
    """After every GPU test, the kernels' status word must be clean."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from elastikernel_b200 import _lib

    st = _lib.device_status(0, clear=True)
    assert st == 0, f"kernel status word = {st:#x} (bounded wait timed out or bad index)"
