"""GPU parity of the GEMM kernels (tcgen05 bf16 path, the fp32 path through split bf16
products on the tensor cores, and the SIMT path)
against the oracle, the golden fixtures and the reference's known answers.
Tolerances: tests/_tol.py.  fp32 outputs: the stated 1e-4 on the output's own
scale, |got - ref| <= 1e-4 * max(|ref|, rms(ref)) against the float64 product
(a TF32 product fails it), plus 1e-4 of the |A||B| condition; bf16 outputs:
1e-2 relative with a 1e-2*rms floor for entries that cancel to ~0."""
import ctypes
from pathlib import Path

import numpy as np
import pytest

from tests._tol import assert_dot_close, assert_output_close, assert_rel
from oracle.oracle import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def stream(torch):
    return torch.cuda.current_stream().cuda_stream


def status_word():
    from bee_b200 import _capi
    code = ctypes.c_int(-1)
    _capi.call("bee_b200_device_status", ctypes.byref(code))
    return code.value


def run_bmm(torch, a_bits, b_bits, batch, m, k, n, b_trans=False, out_f32=False, alpha=1.0):
    from bee_b200 import _capi
    da = torch.from_numpy(np.ascontiguousarray(a_bits).view(np.int16)).cuda()
    db = torch.from_numpy(np.ascontiguousarray(b_bits).view(np.int16)).cuda()
    dc = torch.empty(batch * m * n, dtype=torch.float32 if out_f32 else torch.int16, device="cuda")
    _capi.call("bee_b200_bmm", _capi.BF16, _capi.F32 if out_f32 else _capi.BF16, da.data_ptr(), db.data_ptr(),
               dc.data_ptr(), batch, m, k, n, int(b_trans), float(alpha), stream(torch))
    torch.cuda.synchronize()
    assert status_word() == 0, "a tensor-core pipeline wait gave up"
    c = dc.cpu().numpy()
    return (c if out_f32 else bf16_bits_to_f32(c.view(np.uint16))).reshape(batch, m, n)


def f64_product(a, b):
    return np.asarray(a, np.float64) @ np.asarray(b, np.float64)


def rand_bf16(rng, shape, scale=1.0):
    return f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


# ---------------------------------------------------------------- fp32 (SIMT below 2^28 multiply-adds, split bf16 on the tensor cores above)

def test_matmul_f32_kat(cuda):
    """Tests/Tensor/MatmulTests.cpp:31-62."""
    from bee_b200 import _capi
    torch = cuda
    a = torch.tensor([[1, 2], [3, 4]], dtype=torch.float32, device="cuda")
    b = torch.tensor([[5, 6], [7, 8]], dtype=torch.float32, device="cuda")
    c = torch.empty(2, 2, dtype=torch.float32, device="cuda")
    _capi.call("bee_b200_matmul", _capi.F32, a.data_ptr(), b.data_ptr(), c.data_ptr(), 2, 2, 2, stream(torch))
    torch.cuda.synchronize()
    assert c.cpu().tolist() == [[19, 22], [43, 50]]


@pytest.mark.parametrize("name", ["matmul_f32_17x13x11", "matmul_f32_33x65x47", "matmul_f32_128x96x160"])
def test_matmul_f32_golden(cuda, name):
    from bee_b200 import _capi
    torch = cuda
    g = load(name)
    m, k = g["a"].shape
    n = g["b"].shape[1]
    a, b = torch.from_numpy(g["a"]).cuda(), torch.from_numpy(g["b"]).cuda()
    c = torch.empty(m, n, dtype=torch.float32, device="cuda")
    _capi.call("bee_b200_matmul", _capi.F32, a.data_ptr(), b.data_ptr(), c.data_ptr(), m, k, n, stream(torch))
    torch.cuda.synchronize()
    got = c.cpu().numpy()
    assert_output_close(got, f64_product(g["a"], g["b"]), 1e-4, what=name)
    assert_dot_close(got, g["c"], g["a"], g["b"], 1e-4, what=name)


def test_matmul_f32_1024_config(cuda, oracle):
    """Config: fp32 C = A.B, M = N = K = 1024, A, B uniform[-1, 1), rel tol 1e-4."""
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(1024)
    a = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    b = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c = torch.empty(1024, 1024, dtype=torch.float32, device="cuda")
    _capi.call("bee_b200_matmul", _capi.F32, da.data_ptr(), db.data_ptr(), c.data_ptr(), 1024, 1024, 1024,
               stream(torch))
    torch.cuda.synchronize()
    got = c.cpu().numpy()
    assert_output_close(got, f64_product(a, b), 1e-4, what="fp32 1024^3")
    assert_dot_close(got, oracle.matmul_f32(a, b), a, b, 1e-4, what="fp32 1024^3")


def _matmul_f32(torch, a, b):
    from bee_b200 import _capi
    (m, k), n = a.shape, b.shape[1]
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c = torch.full((m, n), 7.0, dtype=torch.float32, device="cuda")
    _capi.call("bee_b200_matmul", _capi.F32, da.data_ptr(), db.data_ptr(), c.data_ptr(), m, k, n, stream(torch))
    torch.cuda.synchronize()
    return c.cpu().numpy()


# Shapes on the tensor-core fp32 path (K and N multiples of 8, M*N*K >= 2^28); by
# their tile counts they run on 256x256 pair tiles in one batch (2304 x 2304), or on
# 128x128 tiles in one, two, three or six batches of products (1024^3 above: two).
@pytest.mark.parametrize("m,k,n,spread", [(2304, 64, 2304, 0), (1024, 256, 2048, 0), (128, 16384, 128, 0),
                                          (2048, 64, 2048, 0), (600, 512, 1024, 0), (1024, 256, 1024, 30)])
def test_matmul_f32_split_path(cuda, oracle, m, k, n, spread):
    """fp32 matmul through the three-piece bf16 split on the tensor cores against
    the oracle, 1e-4 of |A||B|; spread > 0 scales the entries by 2^-spread..2^spread."""
    torch = cuda
    rng = np.random.default_rng(m * 7 + k * 3 + n + spread)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    if spread:
        a *= np.exp2(rng.integers(-spread, spread + 1, (m, k))).astype(np.float32)
        b *= np.exp2(rng.integers(-spread, spread + 1, (k, n))).astype(np.float32)
    got = _matmul_f32(torch, a, b)
    assert_output_close(got, f64_product(a, b), 1e-4, what=f"fp32 {m}x{k}x{n} spread {spread}")
    assert_dot_close(got, oracle.matmul_f32(a, b), a, b, 1e-4, what=f"fp32 {m}x{k}x{n} spread {spread}")


def test_matmul_f32_split_nonfinite(cuda, oracle):
    """Infinities, NaNs and values beyond bf16's range in A and B: the outputs of
    the rows and columns that hold them are recomputed in plain fp32, so the
    NaN / +inf / -inf pattern equals the oracle's and the finite entries stay
    within 1e-4 of |A||B|."""
    torch = cuda
    rng = np.random.default_rng(77)
    m, k, n = 512, 1024, 512
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    a[3, 10] = np.inf
    a[7, 20] = 3.39e38
    a[9, 0] = np.nan
    b[5, 5] = -np.inf
    b[100, 9] = np.nan
    b[17, 33] = -3.2e38
    got = _matmul_f32(torch, a, b)
    want = oracle.matmul_f32(a, b)
    for f in (np.isnan, np.isposinf, np.isneginf):
        assert np.array_equal(f(got), f(want)), f"{f.__name__} pattern differs"
    with np.errstate(invalid="ignore", over="ignore"):
        scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    ok = np.isfinite(want) & np.isfinite(scale)
    err = np.abs(got[ok].astype(np.float64) - want[ok]) / np.maximum(scale[ok], 1e-30)
    assert err.max() <= 1e-4, f"finite entries: max error {err.max():.3e} x (|A||B|)"
    with np.errstate(invalid="ignore", over="ignore"):
        want64 = f64_product(a, b)
    ok64 = ok & np.isfinite(want64)
    assert_output_close(got[ok64], want64[ok64], 1e-4, what="fp32 non-finite pattern, finite entries")


@pytest.mark.parametrize("dt,np_t", [("float64", np.float64), ("int32", np.int32), ("int64", np.int64)])
def test_matmul_other_dtypes(cuda, dt, np_t):
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(3)
    m, k, n = 37, 53, 29
    if np.issubdtype(np_t, np.integer):
        a = rng.integers(-20, 20, (m, k)).astype(np_t)
        b = rng.integers(-20, 20, (k, n)).astype(np_t)
    else:
        a = rng.standard_normal((m, k)).astype(np_t)
        b = rng.standard_normal((k, n)).astype(np_t)
    code = {"float64": _capi.F64, "int32": _capi.I32, "int64": _capi.I64}[dt]
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c = torch.empty(m, n, dtype=getattr(torch, dt), device="cuda")
    _capi.call("bee_b200_matmul", code, da.data_ptr(), db.data_ptr(), c.data_ptr(), m, k, n, stream(torch))
    torch.cuda.synchronize()
    want = a @ b
    if np.issubdtype(np_t, np.integer):
        np.testing.assert_array_equal(c.cpu().numpy(), want)
    else:
        np.testing.assert_allclose(c.cpu().numpy(), want, rtol=1e-12, atol=1e-12)


# ---------------------------------------------------------------- bf16 (tcgen05)

@pytest.mark.parametrize("m,k,n", [(128, 64, 128), (128, 64, 256), (256, 128, 512), (300, 200, 264), (7, 8, 8),
                                   (129, 72, 136), (1024, 1024, 1024)])
def test_bf16_gemm_oracle(cuda, oracle, m, k, n):
    torch = cuda
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a = rand_bf16(rng, (m, k))
    b = rand_bf16(rng, (k, n))
    got = run_bmm(torch, a, b, 1, m, k, n)[0]
    assert_rel(got, oracle.bmm_bf16(a, b)[0], 1e-2, floor=1e-2, what=f"bf16 gemm {m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n", [(128, 64, 128), (200, 136, 320), (64, 128, 2048)])
def test_bf16_gemm_b_transposed_f32_out(cuda, oracle, m, k, n):
    torch = cuda
    rng = np.random.default_rng(k + n)
    a = rand_bf16(rng, (m, k))
    bt = rand_bf16(rng, (n, k))  # B stored [N, K]
    got = run_bmm(torch, a, bt, 1, m, k, n, b_trans=True, out_f32=True, alpha=0.125)[0]
    want = oracle.bmm_bf16(a, bt, b_trans=True, alpha=0.125)[0]
    af, bf = bf16_bits_to_f32(a), bf16_bits_to_f32(bt).T
    assert_output_close(got, 0.125 * f64_product(af, bf), 1e-4, what="bf16 gemm fp32 out")
    assert_dot_close(got, want, af * 0.125, bf, 1e-4, what="bf16 gemm fp32 out")


@pytest.mark.parametrize("m,k,n,b_trans,out_f32", [(128, 4096, 4096, False, False), (64, 8192, 2048, False, True),
                                                    (96, 2048, 1024, True, True), (128, 3072, 8192, True, False),
                                                    (256, 2048, 256, False, False)])
def test_bf16_gemm_k_split(cuda, m, k, n, b_trans, out_f32):
    """Outputs too small to fill the GPU with long K run as K chunks (fp32
    partials summed in chunk order): against float64 on the output's own scale,
    fp32 output at 1e-4, bf16 output at 1e-2."""
    torch = cuda
    rng = np.random.default_rng(m + k + n)
    a = rand_bf16(rng, (m, k))
    b = rand_bf16(rng, (n, k) if b_trans else (k, n))
    got = run_bmm(torch, a, b, 1, m, k, n, b_trans=b_trans, out_f32=out_f32, alpha=0.5)[0]
    af = bf16_bits_to_f32(a)
    bf = bf16_bits_to_f32(b).T if b_trans else bf16_bits_to_f32(b)
    want = 0.5 * f64_product(af, bf)
    assert_output_close(got, want, 1e-4 if out_f32 else 1e-2, what=f"bf16 gemm K split {m}x{k}x{n}")


def test_bf16_bmm_batched(cuda, oracle):
    torch = cuda
    rng = np.random.default_rng(77)
    batch, m, k, n = 3, 160, 192, 128
    a = rand_bf16(rng, (batch, m, k))
    b = rand_bf16(rng, (batch, k, n))
    got = run_bmm(torch, a, b, batch, m, k, n)
    assert_rel(got, oracle.bmm_bf16(a, b), 1e-2, floor=1e-2, what="batched bf16")
    bt = rand_bf16(rng, (batch, n, k))
    got = run_bmm(torch, a, bt, batch, m, k, n, b_trans=True, out_f32=True)
    assert_rel(got, oracle.bmm_bf16(a, bt, b_trans=True), 1e-4, floor=1e-2, what="batched bf16 b^T")


def test_bf16_gemm_simt_fallback_shapes(cuda, oracle):
    """K not a multiple of 8 cannot be described to TMA: the SIMT path answers."""
    torch = cuda
    rng = np.random.default_rng(13)
    m, k, n = 33, 13, 21
    a = rand_bf16(rng, (m, k))
    b = rand_bf16(rng, (k, n))
    got = run_bmm(torch, a, b, 1, m, k, n)[0]
    assert_rel(got, oracle.bmm_bf16(a, b)[0], 1e-2, floor=1e-2, what="simt fallback")


def test_bf16_gemm_8192_config_sampled(cuda):
    """Config: bf16 C = A.B, M = N = K = 8192, A, B ~ N(0, 1/sqrt(8192)), fp32
    accumulate, bf16 out.  Checked on 96 sampled rows against float64."""
    from bee_b200 import _capi
    torch = cuda
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(8192)
    a = (torch.randn(n, n, device="cuda", generator=g) * (1.0 / np.sqrt(n)) ** 0.5).to(torch.bfloat16)
    b = (torch.randn(n, n, device="cuda", generator=g) * (1.0 / np.sqrt(n)) ** 0.5).to(torch.bfloat16)
    c = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
    _capi.call("bee_b200_bmm", _capi.BF16, _capi.BF16, a.data_ptr(), b.data_ptr(), c.data_ptr(), 1, n, n, n, 0, 1.0,
               stream(torch))
    torch.cuda.synchronize()
    assert status_word() == 0
    rows = np.random.default_rng(1).choice(n, 96, replace=False)
    ah = a[rows].float().cpu().numpy().astype(np.float64)
    bh = b.float().cpu().numpy().astype(np.float64)
    want = ah @ bh
    got = c[rows].float().cpu().numpy()
    assert_rel(got, want, 1e-2, floor=1e-2, what="bf16 8192^3 sampled rows")


def test_bf16_gemm_rejects_mismatched_output(cuda):
    from bee_b200 import _capi
    torch = cuda
    x = torch.empty(64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_capi.BeeError):
        _capi.call("bee_b200_bmm", _capi.BF16, _capi.I32, x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 8, 8, 8, 0,
                   1.0, stream(torch))
