"""Shared pytest configuration: the `gpu` marker and repository import path."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fast_infer_b200 import _lib
    _lib.load()
    return torch.device("cuda:0")


@pytest.fixture()
def device_checks():
    from fast_infer_b200._runtime import device_checks as ctx
    with ctx(True):
        yield
