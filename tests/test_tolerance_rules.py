"""The stated tolerances can tell a correct result from a wrong one.

The fp32 GEMM parity config (1024^3, uniform[-1, 1)) exists to prove 1e-4
relative on the output's own scale; a TF32 product (inputs rounded to a 10-bit
mantissa, as a TF32 tensor-core kernel would) must fail that bound while an
fp32 product passes.  Likewise the attention bound, 1e-2 of max(|O|, rms(O)),
must pass a bf16-rounded output and fail one a few percent off.  The mistakes
are planted on the CPU, in products computed here with numpy.
"""
import numpy as np
import pytest

from tests._tol import assert_output_close, output_err


def _tf32(x):
    """Round fp32 to TF32 (10 explicit mantissa bits), nearest-even."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    keep = ((b >> 13) & 1) + 0xFFF
    return ((b + keep) & ~np.uint64(0x1FFF)).astype(np.uint32).view(np.float32)


def _bf16(x):
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    keep = ((b >> 16) & 1) + 0x7FFF
    return ((b + keep) & ~np.uint64(0xFFFF)).astype(np.uint32).view(np.float32)


def test_fp32_gemm_bound_rejects_tf32():
    rng = np.random.default_rng(1024)
    a = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    b = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    fp32 = a @ b  # fp32 products accumulated in fp32
    assert output_err(fp32, exact) < 1e-5
    assert_output_close(fp32, exact, 1e-4, what="fp32 product")
    tf32 = _tf32(a).astype(np.float64) @ _tf32(b).astype(np.float64)
    assert output_err(tf32, exact) > 1e-4
    with pytest.raises(AssertionError):
        assert_output_close(tf32, exact, 1e-4, what="TF32 product")


def test_attention_bound_rejects_a_few_percent():
    rng = np.random.default_rng(2048)
    heads, seq, hd = 2, 512, 128
    q, k, v = (_bf16(rng.standard_normal((heads, seq, hd)).astype(np.float32)).astype(np.float64) for _ in range(3))
    s = np.einsum("hid,hjd->hij", q, k) / np.sqrt(hd)
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = p @ v
    assert_output_close(_bf16(o.astype(np.float32)), o, 1e-2, what="bf16-rounded output")
    for off in (1.015, 1.03):  # a uniformly wrong output fails the norm-wise bound
        with pytest.raises(AssertionError):
            assert_output_close(o * off, o, 1e-2, what=f"{off - 1:.1%} off", elementwise_rtol=2e-2)
    # what a bf16 tensor-core kernel does: P = exp(s - max) rounded to bf16 before
    # P.V, the row sum l in fp32, the output rounded to bf16 -- inside the bound,
    # but single entries come within ~20% of 1e-2 of rms(O), hence the attention
    # tests' element-wise bound of 2e-2 beside the norm-wise 1e-2
    pb = _bf16(np.exp(s).astype(np.float32)).astype(np.float64)
    l = np.exp(s).sum(-1, keepdims=True)
    got = _bf16(((pb @ v) / l).astype(np.float32))
    assert output_err(got, o) > 5e-3
    assert_output_close(got, o, 1e-2, what="bf16 P", elementwise_rtol=2e-2)
