"""bee_b200: a B200 (sm_100a) backend for the Bee::Tensor compute path.

The product is the C ABI in ``include/bee_b200.h`` implemented by
``bee_b200/_lib/libbee_b200.so`` (hand-written CUDA for sm_100a) and the C++
bridge in ``bee_b200/host`` that re-implements ``bee::tensor::cuda`` over it.
``bee_b200.tensor_cuda`` is the same bridge for Python callers holding torch
tensors.
"""
from ._capi import ABS, ADD, BF16, BOOL, DIV, EXP, F16, F32, F64, I8, I32, I64, LOG, MAX, MIN, MUL, NEG, PROD, SQRT, \
    SUB, SUM, U8, BeeError, LIB_PATH  # noqa: F401

__all__ = ["BeeError", "LIB_PATH"]
