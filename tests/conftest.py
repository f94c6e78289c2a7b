"""Shared pytest configuration: the `gpu` marker and import path."""

import sys

import pytest
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200, sm_100a) and the built extension"
    )


@pytest.fixture(autouse=True)
def _device_status(request):
    """After every GPU test: no bounded tensor-core wait may have given up."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from mamba4_b200 import _lib

    torch.cuda.synchronize()
    assert _lib.load().m4_device_status() == 0, "a tensor-core wait timed out (device status M4_ERR_TIMEOUT)"
