"""Test configuration: registers the `gpu` marker and builds libmuse_proj.so once when stale."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session", autouse=True)
def _built_library():
    from muse_bf16_proj_b200 import build
    build.build()  # no-op unless a source is newer than the library
    yield


def gpu_available() -> bool:
    import torch
    return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10
