"""Test configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs on any machine (library loading, exported symbols, the
oracle against its fixtures and numpy restatements, host-side logic, gloo
data-parallel logic).  `-m gpu` needs a B200 and runs the parity tests
through the C-ABI and through the `ocl` device.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built extension")


@pytest.fixture(scope="session")
def ocl():
    """The imported backend package; the GPU tests require a visible device."""
    import torch

    import pytorch_vulkan_b200 as pkg

    if not torch.ocl.is_available():
        pytest.fail("no ocl (CUDA) device visible; -m gpu tests need a B200")
    return pkg


@pytest.fixture()
def math_fp32(ocl):
    """Run a test with exact-fp32 contractions (SIMT), restoring the mode after."""
    import torch

    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(1)
    yield
    torch.ocl.set_math_mode(old)
