"""The drop-in Tensor library (the reference's Tensor sources compiled with
BEE_TENSOR_WITH_CUDA, its CUDA boundary bee_b200/tensor/Backend.cpp, the new
ops of bee_b200/tensor/Nn.cpp) builds, exports the boundary, and its new ops'
CPU paths give the known answers: tests/cpp/test_bee_tensor_cuda.cpp in `cpu`
mode, no GPU involved."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "oracle" / "_ref"
BIN = REF / "test_bee_tensor_cuda"
LIB = REF / "libbee_tensor_cuda.so"

pytestmark = pytest.mark.skipif(not BIN.exists(), reason="drop-in Tensor library not built (make -C oracle tensor-cuda)")


def test_new_ops_cpu_paths():
    r = subprocess.run([str(BIN), "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "3 of 3 cases passed" in r.stdout


def test_library_implements_the_boundary_with_bee_b200():
    """Every bee::tensor::cuda function of Bee/Tensor/Cuda/Backend.hpp is defined
    in the library, and the library links libbee_b200.so (not Bee::CUDA)."""
    syms = subprocess.run(["nm", "-D", "-C", "--defined-only", str(LIB)], capture_output=True, text=True).stdout
    for fn in ["allocate", "deallocate", "memcpy_h2d", "memcpy_d2h", "memcpy_d2d", "memset", "ew_binary", "ew_unary",
               "ew_cast", "reduce_global", "reduce_axis", "scale_fp", "matmul", "transpose_2d", "random_uniform",
               "random_normal", "random_int", "synchronize", "softmax_rows", "rms_norm_rows", "rope",
               "rms_norm_rope", "bmm", "attention", "strided_copy"]:
        assert f"bee::tensor::cuda::{fn}(" in syms, fn
    for op in ["softmax(", "rms_norm(", "rope(", "rms_norm_rope(", "bmm(", "attention("]:
        assert f"bee::{op}" in syms, op
    needed = subprocess.run(["readelf", "-d", str(LIB)], capture_output=True, text=True).stdout
    assert "libbee_b200.so" in needed
