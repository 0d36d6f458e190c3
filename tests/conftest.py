"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any host (oracle pinning, host logic, C-ABI exports);
`-m gpu` needs a B200 and calls the CUDA library through its C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("sam3.c_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import sam3cu
    sam3cu.init(torch.cuda.current_device())
    return torch.device("cuda")

