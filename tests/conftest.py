"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked ``gpu`` need a B200 (sm_100a) and call the CUDA kernels through
the C ABI; everything else runs on CPU only (oracle pins, host-side argument
validation, ABI export checks, multi-rank host logic over gloo).
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU; runs the CUDA kernels through the C ABI")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, reference_available
    if not reference_available():
        pytest.skip("reference CPU library (oracle/_ref) not built")
    return Reference()


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device and the bee_b200 library loaded (GPU tests only)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from bee_b200 import _capi
    _capi.lib()
    return torch
