"""The FMA-pipe 2^x of the attention softmax meets its stated error bound.

`ex2_fma_x2` in bee_b200/csrc/attention.cu computes a quarter of the softmax
exponentials without the MUFU: x is clamped at -126, split as n = floor(x)
(x + 1.5 * 2^23 rounded toward -inf, so n sits in the low mantissa bits) and
f = x - n in [0, 1); 2^f comes from a cubic fitted for minimum relative error on
[0, 1]; n is added to the exponent field of the cubic's bits.  This test reads
the four coefficients from the source, replays the same steps in float32 (a
separate multiply and add per Horner step, against the kernel's fused ones:
both stay far inside the bound) and checks the stated bound, 7.5e-5 relative,
against float64 2^x, plus the edge behaviour the clamp is there for: no
negative, infinite or NaN result down to x = -1000.
"""
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "bee_b200" / "csrc" / "attention.cu"


def _coefficients():
    body = SRC.read_text()
    fn = body[body.index("__device__ __forceinline__ void ex2_fma_x2"):]
    fn = fn[: fn.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"pack_f32x2\(([0-9.]+)f, \1f\)", fn)]
    assert vals[0] == 12582912.0, vals  # the rounding constant 1.5 * 2^23 comes first
    vals = vals[1:]
    assert len(vals) == 4, vals  # c3, c2, c1, c0 in the order the Horner steps use them
    return np.float32(vals[0]), np.float32(vals[1]), np.float32(vals[2]), np.float32(vals[3])


def _ex2_cubic(x):
    c3, c2, c1, c0 = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)  # 1.5 * 2^23
    n = np.floor(x).astype(np.float32)  # what x + magic rounded toward -inf leaves, minus magic
    t_bits = (magic + n).astype(np.float32).view(np.uint32).astype(np.uint64)
    f = (x - n).astype(np.float32)
    q = (c3 * f + c2).astype(np.float32)
    q = (q * f + c1).astype(np.float32)
    q = (q * f + c0).astype(np.float32)
    bits = (q.view(np.uint32).astype(np.uint64) + ((t_bits << 23) & 0xFFFFFFFF)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_cubic_relative_error_bound():
    x = np.linspace(-125.0, 9.0, 1_000_001, dtype=np.float32)
    got = _ex2_cubic(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 7.5e-5 * 1.02, rel.max()  # the bound stated in the source, float32 rounding on top
    # and tighter than the bf16 rounding of P that follows it by more than an order of magnitude
    assert rel.max() < 2.0 ** -9 / 20


def test_cubic_underflow_is_harmless():
    x = np.concatenate([np.linspace(-1000.0, -120.0, 100_001, dtype=np.float32),
                        np.float32([-np.inf, -126.0, -125.5])])
    got = _ex2_cubic(x)
    assert np.all(np.isfinite(got)) and np.all(got >= 0.0)
    assert got.max() <= np.float32(2.0 ** -119)  # all of them round to ~0 next to any kept probability
