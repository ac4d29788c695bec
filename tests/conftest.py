"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any machine (oracle, host logic, library loading);
`-m gpu` needs a B200 and exercises the CUDA kernels through the C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gpu-kernels_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import build_oracle, oracle as o
    build_oracle.build()
    return o


@pytest.fixture(scope="session")
def nv():
    """The product package with its library loaded; fails loudly when absent."""
    import nvfp4_b200
    nvfp4_b200.lib()
    return nvfp4_b200


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"needs an sm_100 device, found compute capability {major}.x")
    return torch.device("cuda", 0)
