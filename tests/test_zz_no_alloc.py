"""bee_b200_reduce_global_noalloc against bee_b200_reduce_global.

The allocation-free variant serves callers that must not allocate device
memory while they reduce (after an out-of-memory failure, inside a runtime that
owns all device memory, in a loop that must not grow the memory pool).  It must
give the same answers as the allocating entry point, call after call, since
every call reuses one fixed scratch array.  This file is collected last so a
stop-at-first-failure run has already run every other test.
"""
import numpy as np
import pytest

from tests._tol import assert_sum_close

pytestmark = pytest.mark.gpu


def _reduce(torch, name, op, code, x, out):
    from bee_b200 import _capi
    _capi.call(name, op, code, x.data_ptr(), out.data_ptr(), x.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.clone().cpu().numpy()[0]


@pytest.mark.parametrize("n", [1, 257, (1 << 20) + 3, 8192 * 8192])
def test_noalloc_int32_sum_matches_allocating_entry(cuda, n):
    from bee_b200 import _capi
    torch = cuda
    x = torch.from_numpy(np.random.default_rng(n).integers(-1000, 1001, n).astype(np.int32)).cuda()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = _reduce(torch, "bee_b200_reduce_global", 0, _capi.I32, x, out)
    for _ in range(2):  # two calls in a row share the fixed scratch
        out.fill_(12345)
        assert _reduce(torch, "bee_b200_reduce_global_noalloc", 0, _capi.I32, x, out) == want


@pytest.mark.parametrize("op", [0, 1, 2])
def test_noalloc_fp32_matches_allocating_entry(cuda, op):
    from bee_b200 import _capi
    torch = cuda
    xh = np.random.default_rng(op).standard_normal(3_000_017).astype(np.float32)
    x = torch.from_numpy(xh).cuda()
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    want = _reduce(torch, "bee_b200_reduce_global", op, _capi.F32, x, out)
    for _ in range(2):
        out.fill_(-1.0)
        got = _reduce(torch, "bee_b200_reduce_global_noalloc", op, _capi.F32, x, out)
        if op == 0:
            assert_sum_close(got, want, np.abs(xh).sum(), 1e-4, "fp32 sum")
        else:
            assert got == want


def _pool_attr(rt, pool, attr):
    err, v = rt.cudaMemPoolGetAttribute(pool, attr)
    assert err == rt.cudaError_t.cudaSuccess, err
    return int(v)


def test_noalloc_allocates_nothing(cuda):
    """After the warm-up call, further calls (on new streams, where the
    allocating entry point would take new scratch) take nothing from the
    device's stream-ordered pool, the one every allocation of this library comes
    from, and do not lower the device's free memory; the same check does see an
    allocation from that pool."""
    from cuda.bindings import driver as drv
    from cuda.bindings import runtime as rt

    from bee_b200 import _capi
    torch = cuda
    dev = torch.cuda.current_device()
    err, pool = rt.cudaDeviceGetDefaultMemPool(dev)
    assert err == rt.cudaError_t.cudaSuccess, err
    used_now, used_high = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh
    x = torch.from_numpy(np.random.default_rng(5).integers(-1000, 1001, 4 << 20).astype(np.int32)).cuda()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = int(x.sum().item())
    assert _reduce(torch, "bee_b200_reduce_global_noalloc", 0, _capi.I32, x, out) == want  # warm-up
    torch.cuda.synchronize()
    base = _pool_attr(rt, pool, used_now)
    err, = rt.cudaMemPoolSetAttribute(pool, used_high, drv.cuuint64_t(0))  # high-water mark := current use
    assert err == rt.cudaError_t.cudaSuccess, err
    streams = [torch.cuda.Stream() for _ in range(3)]  # new streams: the allocating entry would take new scratch
    for s in streams:
        with torch.cuda.stream(s):
            out.fill_(7)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for s in streams:
        with torch.cuda.stream(s):
            out.fill_(7)
            _capi.call("bee_b200_reduce_global_noalloc", 0, _capi.I32, x.data_ptr(), out.data_ptr(), x.numel(),
                       s.cuda_stream)
            s.synchronize()
            assert int(out.item()) == want  # read without a device allocation
    torch.cuda.synchronize()
    assert _pool_attr(rt, pool, used_high) == base, "the no-allocation entry point took memory from the pool"
    assert _pool_attr(rt, pool, used_now) == base
    assert torch.cuda.mem_get_info()[0] == free_before
    # the check is live: an allocation from the library's pool shows up in it
    import ctypes
    p = ctypes.c_void_p()
    _capi.call("bee_b200_allocate", ctypes.byref(p), 1 << 20, 256, None)
    _capi.call("bee_b200_deallocate", p, None)
    torch.cuda.synchronize()
    assert _pool_attr(rt, pool, used_high) >= base + (1 << 20)


def test_noalloc_other_dtypes_and_errors(cuda):
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(9)
    for dt, code, arr in [("int64", _capi.I64, rng.integers(-10**12, 10**12, 100_003)),
                          ("uint8", _capi.U8, rng.integers(0, 256, 70_001)),
                          ("float64", _capi.F64, rng.standard_normal(50_001))]:
        x = torch.from_numpy(arr.astype(getattr(np, dt))).cuda()
        out = torch.zeros(1, dtype=getattr(torch, dt), device="cuda")
        op = 2 if dt == "uint8" else 0
        want = _reduce(torch, "bee_b200_reduce_global", op, code, x, out)
        for _ in range(2):
            assert _reduce(torch, "bee_b200_reduce_global_noalloc", op, code, x, out) == want
    with pytest.raises(_capi.BeeError, match="empty"):
        _capi.call("bee_b200_reduce_global_noalloc", 0, _capi.I32, 16, 16, 0, None)
    with pytest.raises(_capi.BeeError, match="U8"):
        _capi.call("bee_b200_reduce_global_noalloc", 0, _capi.U8, x.data_ptr(), out.data_ptr(), 16, None)
