"""Pins the oracle (CPU restatement) to the reference.

Three layers, all CPU-only:
1. known-answer tests copied as values from the reference's own test suite;
2. the golden fixtures in tests/golden/ (outputs of the reference's compiled
   CPU path, made by tests/golden/make_golden.py);
3. when oracle/_ref is built, the live reference on fresh seeded inputs.
"""
from pathlib import Path

import numpy as np
import pytest

from tests._tol import assert_dot_close, assert_rel, assert_scaled, assert_sum_close, attention_scale
from oracle.oracle import bf16_bits_to_f32, f32_to_bf16_bits

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


# ---------------------------------------------------------------- 1. KATs

def test_kat_matmul_2x2(oracle):
    # Tests/Tensor/MatmulTests.cpp:31-62: [[1,2],[3,4]] x [[5,6],[7,8]] = [[19,22],[43,50]]
    a = np.array([[1, 2], [3, 4]], np.float32)
    b = np.array([[5, 6], [7, 8]], np.float32)
    np.testing.assert_array_equal(oracle.matmul_f32(a, b), [[19, 22], [43, 50]])


def test_kat_axis_sums(oracle):
    # Tests/Tensor/ReduceTests.cpp:278-295: arange(12) as 3x4, sum(dim=1) -> {6, 22, 38}
    x = np.arange(12, dtype=np.float32).reshape(3, 4)
    np.testing.assert_array_equal(oracle.reduce_rows_f32(0, x), [6, 22, 38])
    # :432-446: 3x17 of ones, sum(dim=1) == 17 per row
    np.testing.assert_array_equal(oracle.reduce_rows_f32(0, np.ones((3, 17), np.float32)), [17, 17, 17])


def test_kat_global_sums(oracle):
    # Tests/Tensor/ReduceTests.cpp:26-57: 2x3 of 2 -> 12
    assert oracle.sum_f32(np.full(6, 2.0, np.float32)) == 12.0
    assert oracle.reduce_global_i32(0, np.full(6, 2, np.int32)) == 12
    # min / max
    x = np.array([3, -7, 11, 0], np.int32)
    assert oracle.reduce_global_i32(1, x) == -7 and oracle.reduce_global_i32(2, x) == 11


def test_int32_sum_wraps_like_int32(oracle):
    # accumulation in the element type (ReduceCpu.hpp:190-193): wraps mod 2^32
    x = np.array([2**31 - 1, 1, 5], np.int32)
    assert oracle.reduce_global_i32(0, x) == -(2**31) + 5


def test_bf16_rounding_definition(oracle):
    bits = np.array([0x3F800000, 0x3F808000, 0x3F818000, 0x3F80FFFF, 0x7F800000, 0xFF800000,
                     0x7FC00001, 0x00000001, 0x807FFFFF, 0x7F7FFFFF], np.uint32)
    x = bits.view(np.float32)
    want = np.array([0x3F80, 0x3F80, 0x3F82, 0x3F81, 0x7F80, 0xFF80, 0x7FFF, 0x0000, 0x8080, 0x7F80], np.uint16)
    np.testing.assert_array_equal(oracle.cast_f32_bf16(x), want)
    np.testing.assert_array_equal(f32_to_bf16_bits(x), want)
    # round trip of representable values is exact
    r = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    rb = bf16_bits_to_f32(f32_to_bf16_bits(r))
    np.testing.assert_array_equal(f32_to_bf16_bits(rb), f32_to_bf16_bits(r))


# ---------------------------------------------------------------- 2. golden fixtures

@pytest.mark.parametrize("name", ["matmul_f32_17x13x11", "matmul_f32_33x65x47", "matmul_f32_128x96x160"])
def test_golden_matmul(oracle, name):
    g = load(name)
    assert_dot_close(oracle.matmul_f32(g["a"], g["b"]), g["c"], g["a"], g["b"], 1e-4, what=name)


@pytest.mark.parametrize("name,op", [("add_f32", 0), ("mul_f32", 2)])
def test_golden_binary(oracle, name, op):
    g = load(name)
    np.testing.assert_array_equal(oracle.binary(op, g["a"], g["b"]), g["c"])


@pytest.mark.parametrize("shape", ["33x257", "5x4099"])
def test_golden_row_reduce(oracle, shape):
    s = load(f"row_sum_f32_{shape}")
    np.testing.assert_array_equal(oracle.reduce_rows_f32(0, s["x"]), s["y"])  # same sequential fp32 order
    m = load(f"row_max_f32_{shape}")
    np.testing.assert_array_equal(oracle.reduce_rows_f32(2, m["x"]), m["y"])


@pytest.mark.parametrize("n", [1, 31, 32, 256, 257, 4096, (1 << 16) + 3])
def test_golden_int32_sum(oracle, n):
    g = load(f"sum_i32_{n}")
    assert oracle.reduce_global_i32(0, g["x"]) == int(g["y"][0])


@pytest.mark.parametrize("shape", ["16x300", "4x8192"])
def test_golden_softmax(oracle, shape):
    g = load(f"softmax_f32_{shape}")
    assert_rel(oracle.softmax_f32(g["x"]), g["y"], 1e-4, floor=0.0, what="softmax")


def test_golden_rms_norm(oracle):
    g = load("rms_norm_bf16in_8x4096")
    np.testing.assert_array_equal(oracle.rms_norm_f32(g["x"], g["w"], 1e-6), g["y"])


def test_golden_rope(oracle):
    g = load("rope_bf16in_2x4x4x128")
    np.testing.assert_array_equal(oracle.rope_f32(g["x"], 4, 4, 128, 10000.0, 0), g["y"])


def test_golden_attention(oracle):
    g = load("attention_bf16in_2x64x32")
    sc = float(1 / np.sqrt(32.0))
    assert_scaled(oracle.attention_f32(g["q"], g["k"], g["v"], sc), g["o"], attention_scale(g["q"], g["k"], g["v"], sc),
                  1e-4, what="attention")


# ---------------------------------------------------------------- 3. live reference

def test_live_reference_row_ops(oracle, reference):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((64, 3000)).astype(np.float32)
    np.testing.assert_array_equal(oracle.reduce_rows_f32(0, x), reference.reduce_rows_f32(0, x)[0])
    np.testing.assert_array_equal(oracle.reduce_rows_f32(2, x), reference.reduce_rows_f32(2, x)[0])
    assert_rel(oracle.softmax_f32(x), reference.softmax_f32(x)[0], 1e-4, floor=0.0, what="softmax")
    w = (1 + 0.02 * rng.standard_normal(3000)).astype(np.float32)
    np.testing.assert_array_equal(oracle.rms_norm_f32(x, w, 1e-6), reference.rms_norm_f32(x, w, 1e-6)[0])


def test_live_reference_global_and_gemm(oracle, reference):
    rng = np.random.default_rng(8)
    xi = rng.integers(-1000, 1001, 3_000_001).astype(np.int32)  # > 4 MB: the parallel chunked path
    assert oracle.reduce_global_i32(0, xi) == reference.reduce_global_i32(0, xi)[0]
    xf = rng.standard_normal(100_003).astype(np.float32)
    assert_sum_close(oracle.sum_f32(xf), reference.reduce_global_f32(0, xf)[0], np.abs(xf).sum(), 1e-5, "fp32 sum")
    a = rng.uniform(-1, 1, (200, 300)).astype(np.float32)
    b = rng.uniform(-1, 1, (300, 100)).astype(np.float32)
    assert_dot_close(oracle.matmul_f32(a, b), reference.matmul_f32(a, b)[0], a, b, 1e-4, what="gemm")


def test_live_reference_rope_attention(oracle, reference):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((3 * 5, 2 * 64)).astype(np.float32)
    np.testing.assert_array_equal(oracle.rope_f32(x, 5, 2, 64, 500.0, 3), reference.rope_f32(x, 5, 2, 64, 500.0, 3)[0])
    q, k, v = (rng.standard_normal((2, 40, 16)).astype(np.float32) for _ in range(3))
    assert_scaled(oracle.attention_f32(q, k, v, 0.25), reference.attention_f32(q, k, v, 0.25)[0],
                  attention_scale(q, k, v, 0.25), 1e-4, what="attention")
