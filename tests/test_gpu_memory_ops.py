"""GPU parity of the memory-bound kernels against the oracle and the golden
fixtures (tolerances: tests/_tol.py).  Every call goes through the C ABI."""
from pathlib import Path

import numpy as np
import pytest

from tests._tol import assert_rel, assert_scaled, assert_sum_close
from oracle.oracle import bf16_bits_to_f32, bf16_round, f32_to_bf16_bits

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bf16_dev(torch, x_f32):
    """fp32 numpy -> bf16 device tensor holding the RNE-rounded values."""
    bits = f32_to_bf16_bits(x_f32).view(np.int16)
    return dev(torch, bits).view(torch.bfloat16)


def bf16_host(t):
    import torch
    torch.cuda.synchronize()
    return bf16_bits_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))


# ---------------------------------------------------------------- elementwise

@pytest.mark.parametrize("n", [1, 7, 8, 31, 4097, 7 * 1031, 1 << 20])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_binary_f32_exact(cuda, oracle, n, op):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(n * 10 + op)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32) + 0.5
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tc.ew_binary(op, dev(torch, a), dev(torch, b), out)
    np.testing.assert_array_equal(host(out), oracle.binary(op, a, b))


@pytest.mark.parametrize("name,op", [("add_f32", 0), ("mul_f32", 2)])
def test_binary_golden(cuda, name, op):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    g = load(name)
    out = torch.empty(g["a"].shape, dtype=torch.float32, device="cuda")
    tc.ew_binary(op, dev(torch, g["a"]), dev(torch, g["b"]), out)
    np.testing.assert_array_equal(host(out), g["c"])


def test_binary_unaligned_views(cuda, oracle):
    """Buffers that are not 16-byte aligned take the element-wise path."""
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(3)
    a = rng.standard_normal(1001).astype(np.float32)
    b = rng.standard_normal(1001).astype(np.float32)
    da, db = dev(torch, a), dev(torch, b)
    out = torch.zeros(1001, dtype=torch.float32, device="cuda")
    _capi.call("bee_b200_ew_binary", 0, 4, da.data_ptr() + 4, db.data_ptr() + 4, out.data_ptr() + 4, 1000,
               torch.cuda.current_stream().cuda_stream)
    np.testing.assert_array_equal(host(out)[1:], a[1:] + b[1:])


@pytest.mark.parametrize("dt,np_t", [("int32", np.int32), ("int64", np.int64), ("uint8", np.uint8),
                                     ("float64", np.float64)])
def test_binary_other_dtypes(cuda, oracle, dt, np_t):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(5)
    n = 3 * 1024 + 5
    if np.issubdtype(np_t, np.integer):
        a = rng.integers(0 if np_t == np.uint8 else -500, 200, n).astype(np_t)
        b = rng.integers(1, 100, n).astype(np_t)
    else:
        a = rng.standard_normal(n).astype(np_t)
        b = rng.standard_normal(n).astype(np_t)
    for op in (0, 1, 2):
        out = torch.empty(n, dtype=getattr(torch, dt), device="cuda")
        tc.ew_binary(op, dev(torch, a), dev(torch, b), out)
        np.testing.assert_array_equal(host(out), oracle.binary(op, a, b))


def test_binary_bf16(cuda):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(6)
    n = 10_000 + 3
    a = bf16_round(rng.standard_normal(n).astype(np.float32))
    b = bf16_round(rng.standard_normal(n).astype(np.float32))
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    tc.ew_binary(0, bf16_dev(torch, a), bf16_dev(torch, b), out)
    # fp32 sum of two bf16 values, rounded once to bf16 (RNE)
    np.testing.assert_array_equal(bf16_host(out), bf16_round((a + b).astype(np.float32)))


def test_unary_f32(cuda):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(11)
    x = rng.uniform(0.1, 4.0, 5000).astype(np.float32)
    for op, fn, exact in [(0, np.negative, True), (1, np.abs, True), (2, np.sqrt, False), (3, np.exp, False),
                          (4, np.log, False)]:
        out = torch.empty_like(dev(torch, x))
        tc.ew_unary(op, dev(torch, x), out)
        want = fn(x.astype(np.float64))
        if exact:
            np.testing.assert_array_equal(host(out), want.astype(np.float32))
        else:
            assert_rel(host(out), want, 1e-6, floor=0.0, what=f"unary {op}")


# ---------------------------------------------------------------- cast

@pytest.mark.parametrize("n", [1, 7, 8, 9, 1000, (1 << 20) + 5])
def test_cast_f32_bf16_bits(cuda, oracle, n):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 10.0 ** rng.integers(-30, 30, n)).astype(np.float32)
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    tc.ew_cast(dev(torch, x), out)
    torch.cuda.synchronize()
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, oracle.cast_f32_bf16(x))


def test_cast_f32_bf16_specials(cuda, oracle):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    bits = np.array([0x3F800000, 0x3F808000, 0x3F818000, 0x3F80FFFF, 0x7F800000, 0xFF800000, 0x00000001,
                     0x807FFFFF, 0x7F7FFFFF, 0x80000000, 0x7FC00000, 0xFFC00001] * 3, np.uint32)
    x = bits.view(np.float32)
    out = torch.empty(x.size, dtype=torch.bfloat16, device="cuda")
    tc.ew_cast(dev(torch, x), out)
    torch.cuda.synchronize()
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    want = oracle.cast_f32_bf16(x)
    nan = np.isnan(x)
    np.testing.assert_array_equal(got[~nan], want[~nan])
    assert np.isnan(bf16_bits_to_f32(got[nan])).all()


def test_cast_bf16_f32_and_ints(cuda):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(12)
    x = bf16_round(rng.standard_normal(4099).astype(np.float32))
    out = torch.empty(4099, dtype=torch.float32, device="cuda")
    tc.ew_cast(bf16_dev(torch, x), out)
    np.testing.assert_array_equal(host(out), x)
    # float -> int truncates toward zero (static_cast), int -> float exact, -> bool is x != 0
    f = np.array([1.9, -1.9, 0.0, 7.5, -0.4], np.float32)
    oi = torch.empty(5, dtype=torch.int32, device="cuda")
    tc.ew_cast(dev(torch, f), oi)
    np.testing.assert_array_equal(host(oi), [1, -1, 0, 7, 0])
    ob = torch.empty(5, dtype=torch.bool, device="cuda")
    tc.ew_cast(dev(torch, f), ob)
    np.testing.assert_array_equal(host(ob), [True, True, False, True, True])


# ---------------------------------------------------------------- reductions

@pytest.mark.parametrize("shape", ["33x257", "5x4099"])
def test_row_reduce_golden(cuda, shape):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    s = load(f"row_sum_f32_{shape}")
    x = s["x"]
    out = torch.empty(x.shape[0], dtype=torch.float32, device="cuda")
    tc.reduce_axis(0, dev(torch, x), out, x.shape[0], x.shape[1], 1)
    assert_sum_close(host(out), s["y"], np.abs(x).sum(1), 1e-4, "row sum")
    m = load(f"row_max_f32_{shape}")
    tc.reduce_axis(2, dev(torch, m["x"]), out, x.shape[0], x.shape[1], 1)
    np.testing.assert_array_equal(host(out), m["y"])


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (100, 2047), (7, 2048), (8192, 8192)])
def test_row_reduce_oracle(cuda, oracle, rows, cols):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    x = np.random.default_rng(rows + cols).standard_normal((rows, cols)).astype(np.float32)
    dx = dev(torch, x)
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    tc.reduce_axis(0, dx, out, rows, cols, 1)
    assert_sum_close(host(out), oracle.reduce_rows_f32(0, x), np.abs(x).sum(1), 1e-4, "row sum")
    for op in (1, 2):
        tc.reduce_axis(op, dx, out, rows, cols, 1)
        np.testing.assert_array_equal(host(out), oracle.reduce_rows_f32(op, x))


def test_axis_reduce_inner(cuda):
    """Tests/Tensor/ReduceTests.cpp:333-350: arange(12) 3x4, sum(dim=0) -> {12, 15, 18, 21}."""
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    x = np.arange(12, dtype=np.float32).reshape(3, 4)
    out = torch.empty(4, dtype=torch.float32, device="cuda")
    tc.reduce_axis(0, dev(torch, x), out, 1, 3, 4)
    np.testing.assert_array_equal(host(out), [12, 15, 18, 21])
    xi = np.random.default_rng(1).integers(-9, 9, (6, 50, 33)).astype(np.int32)
    oi = torch.empty(6 * 33, dtype=torch.int32, device="cuda")
    tc.reduce_axis(0, dev(torch, xi), oi, 6, 50, 33)
    np.testing.assert_array_equal(host(oi).reshape(6, 33), xi.sum(1))


@pytest.mark.parametrize("n", [1, 31, 32, 256, 257, 4096, (1 << 16) + 3])
def test_int32_sum_golden(cuda, n):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    g = load(f"sum_i32_{n}")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    tc.reduce_global(0, dev(torch, g["x"]), out)
    assert int(host(out)[0]) == int(g["y"][0])


@pytest.mark.parametrize("n", [(1 << 20) + 3, 8192 * 8192])
def test_int32_sum_bit_exact_large(cuda, oracle, n):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    x = np.random.default_rng(n).integers(-1000, 1001, n).astype(np.int32)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    dx = dev(torch, x)
    tc.reduce_global(0, dx, out)
    want = oracle.reduce_global_i32(0, x)
    assert int(host(out)[0]) == want
    # repeated calls: the per-call scratch and the ticket are re-armed
    tc.reduce_global(0, dx, out)
    assert int(host(out)[0]) == want


def test_int32_sum_wraps(cuda):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    x = np.full(1 << 16, 2**31 - 1, np.int32)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    tc.reduce_global(0, dev(torch, x), out)
    w = ((2**31 - 1) * (1 << 16)) % 2**32
    assert int(host(out)[0]) == (w - 2**32 if w >= 2**31 else w)


def test_global_reduce_other(cuda, oracle):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(21)
    x = rng.standard_normal(3_000_017).astype(np.float32)
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    dx = dev(torch, x)
    tc.reduce_global(0, dx, out)
    s1 = float(host(out)[0])
    assert_sum_close(s1, x.astype(np.float64).sum(), np.abs(x).sum(), 1e-5, "fp32 sum")
    tc.reduce_global(0, dx, out)
    assert float(host(out)[0]) == s1, "fp32 global sum must be deterministic"
    for op, want in [(1, x.min()), (2, x.max())]:
        tc.reduce_global(op, dx, out)
        assert float(host(out)[0]) == float(want)
    u = rng.integers(0, 256, 100_001).astype(np.uint8)
    ou = torch.zeros(1, dtype=torch.uint8, device="cuda")
    tc.reduce_global(2, dev(torch, u), ou)
    assert int(host(ou)[0]) == int(u.max())


# ---------------------------------------------------------------- softmax

@pytest.mark.parametrize("shape", ["16x300", "4x8192"])
def test_softmax_golden(cuda, shape):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    g = load(f"softmax_f32_{shape}")
    out = torch.empty(g["x"].shape, dtype=torch.float32, device="cuda")
    tc.softmax_rows(dev(torch, g["x"]), out)
    assert_rel(host(out), g["y"], 1e-4, floor=0.0, what="softmax")


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (5, 301), (64, 1024), (9, 4100), (3, 16384), (2, 40003),
                                       (8192, 8192)])
def test_softmax_oracle(cuda, oracle, rows, cols):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    x = np.random.default_rng(rows * cols).standard_normal((rows, cols)).astype(np.float32) * 3
    out = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    tc.softmax_rows(dev(torch, x), out)
    got = host(out)
    assert_rel(got, oracle.softmax_f32(x), 1e-4, floor=0.0, what="softmax")
    np.testing.assert_allclose(got.astype(np.float64).sum(1), 1.0, rtol=1e-4)


# ---------------------------------------------------------------- RMSNorm / RoPE

def test_rms_norm_golden_bf16(cuda):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    g = load("rms_norm_bf16in_8x4096")
    y = torch.empty(g["x"].shape, dtype=torch.bfloat16, device="cuda")
    tc.rms_norm_rows(bf16_dev(torch, g["x"]), bf16_dev(torch, g["w"]), y, 1e-6)
    assert_rel(bf16_host(y), g["y"], 1e-2, what="rms_norm bf16")


@pytest.mark.parametrize("rows,cols", [(1, 4), (3, 5), (17, 4096), (4, 10000)])
def test_rms_norm_f32(cuda, oracle, rows, cols):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(cols)).astype(np.float32)
    y = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    tc.rms_norm_rows(dev(torch, x), dev(torch, w), y, 1e-6)
    assert_rel(host(y), oracle.rms_norm_f32(x, w, 1e-6), 1e-4, what="rms_norm f32")


def test_rope_golden_bf16(cuda):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    g = load("rope_bf16in_2x4x4x128")
    y = torch.empty(g["x"].shape, dtype=torch.bfloat16, device="cuda")
    tc.rope(bf16_dev(torch, g["x"]), y, 4, 4, 128, 10000.0, 0)
    assert_rel(bf16_host(y), g["y"], 1e-2, what="rope bf16")


@pytest.mark.parametrize("batch,seq,heads,hd,off", [(1, 1, 1, 2, 0), (2, 5, 3, 16, 7), (2, 33, 4, 64, 0),
                                                    (1, 2048, 2, 128, 0), (1, 9, 2, 256, 100)])
def test_rope_f32(cuda, oracle, batch, seq, heads, hd, off):
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    x = np.random.default_rng(seq * hd).standard_normal((batch * seq, heads * hd)).astype(np.float32)
    y = torch.empty(x.shape, dtype=torch.float32, device="cuda")
    tc.rope(dev(torch, x), y, seq, heads, hd, 10000.0, off)
    # rotation of a pair (x1, x2): error scale |x1| + |x2| per output
    want = oracle.rope_f32(x, seq, heads, hd, 10000.0, off)
    xr = x.reshape(batch * seq, heads, hd)
    pair = np.concatenate([np.abs(xr[..., : hd // 2]) + np.abs(xr[..., hd // 2:])] * 2, -1).reshape(x.shape)
    assert_scaled(host(y), want, pair, 1e-4, what="rope f32")


def test_rms_norm_rope_llama_config(cuda, oracle):
    """Config: X [16 x 2048, 4096] bf16 N(0,1), w N(1, 0.02), eps 1e-6, RoPE [16, 2048, 32, 128], theta 1e4."""
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    rng = np.random.default_rng(2048)
    rows, cols, seq, heads, hd = 16 * 2048, 4096, 2048, 32, 128
    x = bf16_round(rng.standard_normal((rows, cols)).astype(np.float32))
    w = bf16_round((1 + 0.02 * rng.standard_normal(cols)).astype(np.float32))
    dx, dw = bf16_dev(torch, x), bf16_dev(torch, w)
    y = torch.empty((rows, cols), dtype=torch.bfloat16, device="cuda")
    tc.rms_norm_rope(dx, dw, y, seq, heads, hd, 1e-6, 10000.0, 0)
    got = bf16_host(y)
    # oracle on a sample of rows spanning every position class (full check of 32k rows is minutes of CPU)
    sel = np.unique(np.concatenate([np.arange(0, rows, 97), [rows - 1]]))
    xs = x[sel]
    ref = oracle.rms_norm_f32(xs, w, 1e-6)
    # RoPE needs each row's own position: run the oracle per selected row
    out = np.empty_like(ref)
    for i, r in enumerate(sel):
        out[i] = oracle.rope_f32(ref[i:i + 1], 1, heads, hd, 10000.0, int(r % seq))[0]
    rr = ref.reshape(len(sel), heads, hd)
    pair = np.concatenate([np.abs(rr[..., : hd // 2]) + np.abs(rr[..., hd // 2:])] * 2, -1).reshape(ref.shape)
    assert_scaled(got[sel], out, pair, 1e-2, what="rms_norm+rope bf16")
    # and the two-kernel path agrees with the fused one
    n = torch.empty_like(y)
    tc.rms_norm_rows(dx, dw, n, 1e-6)
    y2 = torch.empty_like(y)
    tc.rope(n, y2, seq, heads, hd, 10000.0, 0)
    assert_scaled(bf16_host(y2)[sel], out, pair, 1e-2, what="rms_norm then rope bf16")


@pytest.mark.parametrize("cols,heads", [(8192, 64), (2048, 16)])
def test_rms_norm_rope_bf16_row_widths(cuda, oracle, cols, heads):
    """Row widths that take the pipelined kernel at 128 threads (2048 columns, one rotate-half
    pair of chunks per thread) and at 256 threads (8192 columns, two pairs), fused and RoPE
    alone, against the oracle on every row."""
    from bee_b200 import tensor_cuda as tc
    torch = cuda
    batch, seq, hd = 2, 48, 128
    rng = np.random.default_rng(cols)
    rows = batch * seq
    x = bf16_round(rng.standard_normal((rows, cols)).astype(np.float32))
    w = bf16_round((1 + 0.02 * rng.standard_normal(cols)).astype(np.float32))
    dx, dw = bf16_dev(torch, x), bf16_dev(torch, w)
    ref = oracle.rms_norm_f32(x, w, 1e-6)
    want = np.empty_like(ref)
    for r in range(rows):
        want[r] = oracle.rope_f32(ref[r:r + 1], 1, heads, hd, 10000.0, r % seq)[0]
    rr = ref.reshape(rows, heads, hd)
    pair = np.concatenate([np.abs(rr[..., : hd // 2]) + np.abs(rr[..., hd // 2:])] * 2, -1).reshape(ref.shape)
    y = torch.empty((rows, cols), dtype=torch.bfloat16, device="cuda")
    tc.rms_norm_rope(dx, dw, y, seq, heads, hd, 1e-6, 10000.0, 0)
    assert_scaled(bf16_host(y), want, pair, 1e-2, what=f"rms_norm+rope bf16 x{cols}")
    # RoPE alone on the same rows (one pass, no sum of squares)
    y2 = torch.empty_like(y)
    tc.rope(dx, y2, seq, heads, hd, 10000.0, 0)
    want2 = np.empty_like(x)
    for r in range(rows):
        want2[r] = oracle.rope_f32(x[r:r + 1], 1, heads, hd, 10000.0, r % seq)[0]
    xr = x.reshape(rows, heads, hd)
    pair2 = np.concatenate([np.abs(xr[..., : hd // 2]) + np.abs(xr[..., hd // 2:])] * 2, -1).reshape(x.shape)
    assert_scaled(bf16_host(y2), want2, pair2, 1e-2, what=f"rope bf16 x{cols}")


def test_device_selection(cuda):
    import ctypes
    from bee_b200 import _capi
    torch = cuda
    n = ctypes.c_int(-1)
    _capi.call("bee_b200_device_count", ctypes.byref(n))
    assert n.value == torch.cuda.device_count() >= 1
    _capi.call("bee_b200_set_device", 0)
    d = ctypes.c_int(-1)
    _capi.call("bee_b200_get_device", ctypes.byref(d))
    assert d.value == 0
    with pytest.raises(_capi.BeeError):
        _capi.call("bee_b200_set_device", 1000)
    # the failed call leaves no error behind for the next launch
    x = torch.ones(64, device="cuda")
    y = torch.empty_like(x)
    _capi.call("bee_b200_ew_binary", _capi.ADD, _capi.F32, x.data_ptr(), x.data_ptr(), y.data_ptr(), 64,
               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert float(y.sum()) == 128.0
