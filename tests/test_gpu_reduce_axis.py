"""GPU parity of the axis reductions beyond the row reduce: reductions over a
non-innermost dim (column kernel, split over axis segments), few long rows
(split over CTAs), and the integer mean (bee_b200_reduce_mean_int).

Integer sums / products (wrapping) and min / max are order-independent, so
they are compared bit for bit; float sums within 1e-5 (fp32) / 1e-12 (fp64) of
sum |x| against a float64 sum, float products within 2n units of roundoff
relative (n factors); the integer mean bit for bit against the
oracle's restatement of the reference (exact sum, one rounding)."""
import numpy as np
import pytest

from tests._tol import assert_sum_close
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu

NP = {1: np.uint8, 2: np.int32, 3: np.int64, 4: np.float32, 5: np.float64}
OPS = {0: "sum", 1: "min", 2: "max", 3: "prod"}


def data(rng, shape, dt, op):
    if dt == 1:
        return rng.integers(0, 256, size=shape, dtype=np.uint8)
    if dt in (2, 3):
        lo, hi = (-3, 4) if op == 3 else (-1000, 1001)
        return rng.integers(lo, hi, size=shape).astype(NP[dt])
    if op == 3:
        return (1.0 + 0.01 * rng.standard_normal(shape)).astype(NP[dt])
    return rng.standard_normal(shape).astype(NP[dt])


def want(x, op, axis):
    if op == 0:
        return x.sum(axis=axis, dtype=x.dtype) if x.dtype.kind in "iu" else x.astype(np.float64).sum(axis=axis)
    if op == 3:
        return x.prod(axis=axis, dtype=x.dtype) if x.dtype.kind in "iu" else x.astype(np.float64).prod(axis=axis)
    return x.min(axis=axis) if op == 1 else x.max(axis=axis)


def run_axis(torch, op, dt, x, outer, axis, inner, offset_elems=0):
    from bee_b200 import _capi
    xs = torch.from_numpy(np.ascontiguousarray(x).reshape(-1).view(np.uint8).copy()).cuda()
    es = np.dtype(NP[dt]).itemsize
    if offset_elems:
        pad = torch.zeros(offset_elems * es + xs.numel(), dtype=torch.uint8, device="cuda")
        pad[offset_elems * es:] = xs
        xs = pad
    out = torch.zeros(outer * inner * es, dtype=torch.uint8, device="cuda")
    _capi.call("bee_b200_reduce_axis", op, dt, xs.data_ptr() + offset_elems * es, out.data_ptr(), outer, axis, inner,
               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(NP[dt]).reshape(outer, inner)


def check(got, x, op, dt):
    ref = want(x, op, 1)
    if op in (0, 3) and dt in (4, 5):
        if op == 0:
            assert_sum_close(got, ref, np.abs(x.astype(np.float64)).sum(axis=1), 1e-5 if dt == 4 else 1e-12, "sum")
        else:  # a product of n rounded factors: relative error up to about n units of roundoff
            u = 2.0 ** -24 if dt == 4 else 2.0 ** -53
            assert_sum_close(got, ref, np.abs(ref), max(1e-5 if dt == 4 else 1e-12, 2 * x.shape[1] * u), "prod")
    else:
        np.testing.assert_array_equal(got, ref)


COLUMN_SHAPES = [(1, 3, 4), (6, 50, 33), (1, 4096, 1024), (3, 1000, 257), (2, 70000, 8), (128, 64, 128), (1, 5, 3),
                 (4, 129, 12)]


@pytest.mark.parametrize("dt", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("shape", COLUMN_SHAPES, ids=[f"{o}x{a}x{i}" for o, a, i in COLUMN_SHAPES])
def test_column_reduce(cuda, dt, op, shape):
    if dt == 1 and op in (0, 3):
        pytest.skip("U8 supports min / max only (as in the reference)")
    rng = np.random.default_rng(hash((dt, op, shape)) % (2 ** 32))
    x = data(rng, shape, dt, op)
    check(run_axis(cuda, op, dt, x, *shape), x, op, dt)


def test_column_reduce_misaligned_base(cuda):
    """A base pointer off the 16-byte grid takes the element path."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 300, 64)).astype(np.float32)
    check(run_axis(cuda, 0, 4, x, 2, 300, 64, offset_elems=1), x, 0, 4)


@pytest.mark.parametrize("dt", [2, 4])
@pytest.mark.parametrize("outer,axis", [(4, 1 << 18), (2, (1 << 20) + 5), (1, (1 << 20) + 3), (100, 1 << 16)])
def test_few_long_rows(cuda, dt, outer, axis):
    rng = np.random.default_rng(outer + axis)
    for op in (0, 2):
        x = data(rng, (outer, axis, 1), dt, op)
        check(run_axis(cuda, op, dt, x, outer, axis, 1), x, op, dt)


def test_sum_over_rows_8192(cuda):
    """sum(x, 0) of the [8192, 8192] fp32 config (column reduce at full size)."""
    rng = np.random.default_rng(8192)
    x = rng.standard_normal((1, 8192, 8192)).astype(np.float32)
    check(run_axis(cuda, 0, 4, x, 1, 8192, 8192), x, 0, 4)


def run_mean(torch, dt, x, outer, axis, inner):
    from bee_b200 import _capi
    dx = torch.from_numpy(np.ascontiguousarray(x).reshape(-1)).cuda()
    out = torch.zeros(outer * inner, dtype=torch.float64, device="cuda")
    _capi.call("bee_b200_reduce_mean_int", dt, dx.data_ptr(), out.data_ptr(), outer, axis, inner,
               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(outer, inner)


@pytest.mark.parametrize("dt", [2, 3])
@pytest.mark.parametrize("shape", [(1, 1, 1), (1, 31, 1), (1, (1 << 20) + 3, 1), (5, 4099, 1), (3, 1 << 17, 1),
                                   (1, 8192, 8192), (6, 50, 33), (2, 7, 16)])
def test_mean_int(cuda, dt, shape):
    rng = np.random.default_rng(sum(shape) + dt)
    x = rng.integers(-1000, 1001, size=shape).astype(NP[dt])
    if dt == 3:
        x = x * np.int64(1 << 30)  # magnitudes ~2^40: the sums stay exact in double below 2^53
    got = run_mean(cuda, dt, x, *shape)
    ref = Oracle.mean_int(x, axis=1)
    assert np.array_equal(got, ref), f"max diff {np.max(np.abs(got - ref))}"


def test_mean_int_rejects_float(cuda):
    from bee_b200 import _capi
    with pytest.raises(_capi.BeeError, match="I32 or I64"):
        _capi.call("bee_b200_reduce_mean_int", 4, 16, 16, 1, 4, 1, None)
