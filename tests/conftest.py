"""pytest configuration: the `gpu` marker and import paths.

Tests marked ``gpu`` need a B200 (sm_100a) and the built CUDA library; run
them with ``pytest -m gpu``.  Everything else runs on a CPU-only machine.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run it on the GPU box with -m gpu)")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"needs an sm_100 device, found compute capability {major}.x")
    from ferret_b200 import build
    build.build()
    return torch.device("cuda", 0)
