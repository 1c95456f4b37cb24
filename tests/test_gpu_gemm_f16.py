"""GPU parity of the f16-input paths: the tcgen05 GEMM with f16 A and B (fp32
accumulate; f16 or fp32 output), its SIMT fallback, and the f16 casts and
elementwise ops, against IEEE binary16 round-to-nearest-even (numpy's float16)
and float64 products of the same f16 inputs.  Tolerances (tests/_tol.py): f16
outputs 1e-2 relative (1e-2*rms floor) and 1e-2 on the output's own scale; fp32
outputs 1e-4 on the output's own scale; casts and elementwise ops bit-exact."""
import ctypes

import numpy as np
import pytest

from oracle.oracle import f16_bits_to_f32, f32_to_f16_bits, matmul_exact
from tests._tol import assert_output_close, assert_rel

pytestmark = pytest.mark.gpu


def _stream(torch):
    return torch.cuda.current_stream().cuda_stream


def _status():
    from bee_b200 import _capi
    code = ctypes.c_int(-1)
    _capi.call("bee_b200_device_status", ctypes.byref(code))
    return code.value


def _rand_f16(rng, shape, scale=1.0):
    return f32_to_f16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def _bmm_f16(torch, a_bits, b_bits, batch, m, k, n, b_trans=False, out_f32=False, alpha=1.0):
    from bee_b200 import _capi
    da = torch.from_numpy(np.ascontiguousarray(a_bits).view(np.int16)).cuda()
    db = torch.from_numpy(np.ascontiguousarray(b_bits).view(np.int16)).cuda()
    dc = torch.empty(batch * m * n, dtype=torch.float32 if out_f32 else torch.int16, device="cuda")
    _capi.call("bee_b200_bmm", _capi.F16, _capi.F32 if out_f32 else _capi.F16, da.data_ptr(), db.data_ptr(),
               dc.data_ptr(), batch, m, k, n, int(b_trans), float(alpha), _stream(torch))
    torch.cuda.synchronize()
    assert _status() == 0, "a tensor-core pipeline wait gave up"
    c = dc.cpu().numpy()
    return (c if out_f32 else f16_bits_to_f32(c.view(np.uint16))).reshape(batch, m, n)


# (7, 8, 8) and (33, 13, 21) take the SIMT path (too small for a tile / K not a
# multiple of 8); the rest the tcgen05 kernels (1-SM tiles, CTA-pair tiles).
@pytest.mark.parametrize("m,k,n", [(128, 64, 128), (128, 64, 256), (256, 128, 512), (300, 200, 264), (7, 8, 8),
                                   (33, 13, 21), (129, 72, 136), (1024, 1024, 1024)])
def test_f16_gemm_f16_out(cuda, m, k, n):
    torch = cuda
    rng = np.random.default_rng(m * 5 + k * 3 + n)
    a, b = _rand_f16(rng, (m, k)), _rand_f16(rng, (k, n))
    got = _bmm_f16(torch, a, b, 1, m, k, n)[0]
    want = matmul_exact(f16_bits_to_f32(a), f16_bits_to_f32(b))
    assert_rel(got, want, 1e-2, floor=1e-2, what=f"f16 gemm {m}x{k}x{n}")
    assert_output_close(got, want, 1e-2, what=f"f16 gemm {m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n,b_trans", [(128, 64, 128, False), (200, 136, 320, True), (512, 256, 512, False),
                                           (64, 128, 2048, True)])
def test_f16_gemm_f32_out(cuda, m, k, n, b_trans):
    torch = cuda
    rng = np.random.default_rng(k + n + int(b_trans))
    a = _rand_f16(rng, (m, k))
    b = _rand_f16(rng, (n, k) if b_trans else (k, n))
    got = _bmm_f16(torch, a, b, 1, m, k, n, b_trans=b_trans, out_f32=True, alpha=0.25)[0]
    want = matmul_exact(f16_bits_to_f32(a), f16_bits_to_f32(b), b_trans=b_trans, alpha=0.25)
    assert_output_close(got, want, 1e-4, what=f"f16 gemm fp32 out {m}x{k}x{n} b^T={b_trans}")


def test_f16_bmm_batched_and_wide_range(cuda):
    """Batched, and entries up to ~2^8 (f16 keeps 11 bits of mantissa over a
    narrower exponent range than bf16): products stay finite and exact in fp32."""
    torch = cuda
    rng = np.random.default_rng(16)
    batch, m, k, n = 3, 160, 192, 384
    a = f32_to_f16_bits((rng.standard_normal((batch, m, k)) * np.exp2(rng.integers(-8, 9, (batch, m, k))))
                        .astype(np.float32))
    b = _rand_f16(rng, (batch, k, n))
    got = _bmm_f16(torch, a, b, batch, m, k, n, out_f32=True)
    assert_output_close(got, matmul_exact(f16_bits_to_f32(a), f16_bits_to_f32(b)), 1e-4, what="batched f16 fp32 out")


def test_f16_matmul_entry_and_overflow(cuda):
    """bee_b200_matmul(F16) is f16 in, f16 out; outputs beyond f16's range
    round to +-inf as IEEE binary16 does."""
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(3)
    m = k = n = 256
    a = _rand_f16(rng, (m, k))
    b = _rand_f16(rng, (k, n))
    a[0, :] = f32_to_f16_bits(np.full(k, 300.0, np.float32))
    b[:, 0] = f32_to_f16_bits(np.full(k, 300.0, np.float32))  # C[0, 0] = 256 * 9e4, beyond 65504
    da = torch.from_numpy(a.view(np.int16)).cuda()
    db = torch.from_numpy(b.view(np.int16)).cuda()
    dc = torch.empty(m * n, dtype=torch.int16, device="cuda")
    _capi.call("bee_b200_matmul", _capi.F16, da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, k, n, _stream(torch))
    torch.cuda.synchronize()
    got = f16_bits_to_f32(dc.cpu().numpy().view(np.uint16)).reshape(m, n)
    want = matmul_exact(f16_bits_to_f32(a), f16_bits_to_f32(b))
    assert np.isposinf(got[0, 0])
    ok = np.abs(want) < 65504
    assert np.array_equal(np.isinf(got), ~ok)
    assert_rel(got[ok], want[ok], 1e-2, floor=1e-2, what="f16 matmul")


def test_f16_gemm_8192_config_sampled(cuda):
    """The bf16 8192^3 config with f16 inputs: C = A.B, M = N = K = 8192,
    A, B ~ N(0, 1/sqrt(8192)), fp32 accumulate, f16 out; 96 sampled rows
    against float64."""
    from bee_b200 import _capi
    torch = cuda
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(8193)
    a = (torch.randn(n, n, device="cuda", generator=g) * (1.0 / np.sqrt(n)) ** 0.5).to(torch.float16)
    b = (torch.randn(n, n, device="cuda", generator=g) * (1.0 / np.sqrt(n)) ** 0.5).to(torch.float16)
    c = torch.empty(n, n, dtype=torch.float16, device="cuda")
    _capi.call("bee_b200_bmm", _capi.F16, _capi.F16, a.data_ptr(), b.data_ptr(), c.data_ptr(), 1, n, n, n, 0, 1.0,
               _stream(torch))
    torch.cuda.synchronize()
    assert _status() == 0
    rows = np.random.default_rng(2).choice(n, 96, replace=False)
    want = a[rows].double().cpu().numpy() @ b.double().cpu().numpy()
    got = c[rows].float().cpu().numpy()
    assert_rel(got, want, 1e-2, floor=1e-2, what="f16 8192^3 sampled rows")
    assert_output_close(got, want, 1e-2, what="f16 8192^3 sampled rows")


def test_f16_casts_bit_exact(cuda):
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(100_003) * np.exp2(rng.integers(-30, 20, 100_003))).astype(np.float32)
    x[:8] = [0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 6e-8, 2.9e-8]  # max, overflow, subnormal, underflow
    dx = torch.from_numpy(x).cuda()
    h = torch.empty(x.size, dtype=torch.int16, device="cuda")
    _capi.call("bee_b200_ew_cast", _capi.F32, dx.data_ptr(), _capi.F16, h.data_ptr(), x.size, _stream(torch))
    torch.cuda.synchronize()
    assert np.array_equal(h.cpu().numpy().view(np.uint16), f32_to_f16_bits(x))
    back = torch.empty(x.size, dtype=torch.float32, device="cuda")
    _capi.call("bee_b200_ew_cast", _capi.F16, h.data_ptr(), _capi.F32, back.data_ptr(), x.size, _stream(torch))
    torch.cuda.synchronize()
    assert np.array_equal(back.cpu().numpy(), f16_bits_to_f32(f32_to_f16_bits(x)))
    xd = x.astype(np.float64) * (1 + 2.0 ** -30)  # doubles just off f32 values: one rounding from double
    dd = torch.from_numpy(xd).cuda()
    _capi.call("bee_b200_ew_cast", _capi.F64, dd.data_ptr(), _capi.F16, h.data_ptr(), x.size, _stream(torch))
    torch.cuda.synchronize()
    assert np.array_equal(h.cpu().numpy().view(np.uint16), xd.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_f16_binary_bit_exact(cuda, op):
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(op)
    n = 70_001
    a = rng.standard_normal(n).astype(np.float16)
    b = (rng.standard_normal(n) + 3.0).astype(np.float16)
    da, db = (torch.from_numpy(v.view(np.int16)).cuda() for v in (a, b))
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    _capi.call("bee_b200_ew_binary", op, _capi.F16, da.data_ptr(), db.data_ptr(), out.data_ptr(), n, _stream(torch))
    torch.cuda.synchronize()
    f = [np.add, np.subtract, np.multiply, np.divide][op]
    want = f(a.astype(np.float32), b.astype(np.float32)).astype(np.float16)  # fp32 math, one f16 rounding
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))
