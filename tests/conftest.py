"""Shared pytest configuration.

Markers: ``gpu`` -- needs a B200 (sm_100) device; everything else runs on CPU.
The repository root is put on sys.path so tests import ``final_b200`` and the
``oracle`` checker (test infrastructure) directly.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
if os.path.join(ROOT, "oracle") not in sys.path:
    sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA sm_100 (B200) device")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"needs an sm_100 device, found sm_{major}x")
    return torch.device("cuda:0")
