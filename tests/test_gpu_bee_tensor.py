"""bee::* ops on Device::CUDA tensors through the reference's own Tensor layer
built on bee_b200 (the cases of Tests/Tensor/CudaStubTests.cpp:42-571 and the
new ops, tests/cpp/test_bee_tensor_cuda.cpp), against the same ops on the CPU."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BIN = ROOT / "oracle" / "_ref" / "test_bee_tensor_cuda"

pytestmark = pytest.mark.gpu


def test_bee_tensor_ops_on_cuda_match_cpu():
    assert BIN.exists(), "the drop-in Tensor library and its test were not built (make -C oracle tensor-cuda)"
    r = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout
