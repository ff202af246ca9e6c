"""Shared test setup.

Two classes of test, as loom.cpp splits hermetic and hardware tests (tests/CMakeLists.txt:1-18):
  - unmarked: run anywhere (the oracle against the golden vectors, host-side logic, the C-ABI's
    symbols and argument checks, multi-rank logic on gloo);
  - @pytest.mark.gpu: the parity tests proper, through the C-ABI on a CUDA device. They fail (never
    skip) when the library is missing.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("loom.cpp_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the B200 kernels)")


@pytest.fixture(scope="session")
def oracle():
    import oracle_binding

    oracle_binding.lib()
    return oracle_binding


@pytest.fixture(scope="session")
def sel():
    """The product binding, for GPU tests: the library must load and a device must be present."""
    import torch

    import loom_select

    assert torch.cuda.is_available(), "GPU test without a CUDA device"
    loom_select.lib()
    return loom_select


@pytest.fixture(scope="session")
def dev():
    import torch

    return torch.device("cuda", 0)
