"""Test configuration.

* ``-m "not gpu"`` tests run anywhere (oracle vs golden vectors, host logic,
  ABI exports, the backend wiring against fakes).
* ``-m gpu`` tests need a B200 and call the CUDA library through its C ABI.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "vllm-fp8kv_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")


def golden(name):
    import numpy as np

    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)
