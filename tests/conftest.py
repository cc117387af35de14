"""Shared fixtures.  GPU tests are marked ``gpu`` and call the CUDA library through its C ABI;
everything else runs on the CPU (oracle, host logic, library exports)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (run with -m gpu)")


@pytest.fixture(scope="session", autouse=True)
def _native_built():
    """Build (incrementally) the CUDA library and the CPU oracle before any test."""
    from hayai_b200 import _build

    _build.build_all()


@pytest.fixture(scope="session")
def engine():
    """A CudaEngine on cuda:0.  Fails (does not skip) when no GPU is present, so a GPU run
    can never pass on a silent fallback."""
    import torch

    from hayai_b200 import CudaEngine

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.init()
    eng = CudaEngine(0)
    yield eng
    eng.close()
