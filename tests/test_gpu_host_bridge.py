"""Runs the C++ program that exercises the host bridge (bee_b200/host) — the
C++ calls a Bee::Tensor maintainer makes — on the GPU."""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
BIN = Path(__file__).resolve().parent.parent / "bee_b200" / "_lib" / "test_host_bridge"


def test_cpp_host_bridge(cuda):
    assert BIN.exists(), "build the library first (python -m bee_b200.build)"
    r = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "host bridge ok" in r.stdout
