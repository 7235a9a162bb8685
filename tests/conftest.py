"""Shared test setup: import paths, the ``gpu`` marker and small helpers.

Tests marked ``gpu`` run only on a machine with an sm_100 GPU (``pytest -m gpu``); the rest run on
the CPU (``pytest -m "not gpu"``) and never launch a kernel.
"""
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "nn-cpp_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built libnnb.so")


@pytest.fixture(scope="session")
def cuda():
    """torch with a usable CUDA device; the GPU tests fail (not skip) without one."""
    import torch
    assert torch.cuda.is_available(), "gpu-marked test run without a CUDA device"
    torch.cuda.init()
    return torch
