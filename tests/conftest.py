"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on CPU."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built libabft_b200.so")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"the library is built for sm_100a, device is sm_{major}{minor}"
    from vla_abft_estimate_b200 import _native

    _native.lib()  # fails loudly when the library is missing
    return torch.device("cuda", 0)
