"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pk():
    return __graft_entry__.load()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    o.lib()
    return o


@pytest.fixture(scope="session")
def device(pk):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = pk.kernels.Device(0)
    yield dev
    dev.close()


@pytest.fixture(autouse=True)
def _release_device_temporaries(request):
    yield
    if request.node.get_closest_marker("gpu") is not None:
        import gpu_util

        gpu_util.release()
