"""GPU parity of the layout kernels (bee_b200_transpose_2d, bee_b200_strided_copy)
against the oracle's strided gather (numpy index arithmetic restating
contiguous_copy_into, Bee/Tensor/Core/Tensor.cpp:119-147).  Pure data movement:
every comparison is bit-exact."""
import ctypes

import numpy as np
import pytest

from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu

# dtype code -> unsigned numpy dtype of the same size: random bit patterns are
# compared as bits (a float view would hold NaNs, which never compare equal)
DTYPES = {0: np.uint8, 1: np.uint8, 2: np.uint32, 3: np.uint64, 4: np.uint32, 5: np.uint64, 6: np.uint8, 7: np.uint16,
          8: np.uint16}


def rand_bits(rng, n, npdt):
    raw = rng.integers(0, 256, size=n * np.dtype(npdt).itemsize, dtype=np.uint8)
    return raw.view(npdt)


def to_dev(torch, arr):
    t = torch.from_numpy(np.ascontiguousarray(arr).view(np.uint8).copy()).cuda()
    return t


def stream(torch):
    return torch.cuda.current_stream().cuda_stream


def run_transpose(torch, dt, a, rows, cols):
    from bee_b200 import _capi
    npdt = a.dtype
    src = to_dev(torch, a)
    dst = torch.zeros(max(rows * cols * np.dtype(npdt).itemsize, 1), dtype=torch.uint8, device="cuda")
    _capi.call("bee_b200_transpose_2d", dt, src.data_ptr(), dst.data_ptr(), rows, cols, stream(torch))
    torch.cuda.synchronize()
    return dst.cpu().numpy()[: rows * cols * np.dtype(npdt).itemsize].view(npdt)


@pytest.mark.parametrize("dt", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (31, 33), (64, 64), (65, 129), (1000, 3), (3, 1000), (256, 512)])
def test_transpose_2d(cuda, dt, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols + dt)
    a = rand_bits(rng, rows * cols, DTYPES[dt])
    got = run_transpose(cuda, dt, a, rows, cols)
    want = Oracle.strided_gather(a, 0, (cols, rows), (1, cols)).reshape(-1)
    assert np.array_equal(got, want)


def test_transpose_kats(cuda):
    """Tests/CUDA/TransposeTests.cu:79-110."""
    a = np.arange(15, dtype=np.float64) * 0.5
    assert np.array_equal(run_transpose(cuda, 5, a, 3, 5), a.reshape(3, 5).T.reshape(-1))
    b = ((np.arange(32 * 64) % 17) - 8).astype(np.float32) * 0.25
    assert np.array_equal(run_transpose(cuda, 4, b, 32, 64), b.reshape(32, 64).T.reshape(-1))


def test_transpose_misaligned_base_uses_scalar_path(cuda):
    """A base pointer off the 16-byte grid takes the element path on both sides."""
    from bee_b200 import _capi
    torch = cuda
    rows, cols = 70, 90
    rng = np.random.default_rng(9)
    a = rng.standard_normal(rows * cols).astype(np.float32)
    src = torch.zeros(rows * cols + 1, dtype=torch.float32, device="cuda")
    src[1:] = torch.from_numpy(a).cuda()
    dst = torch.zeros(rows * cols + 1, dtype=torch.float32, device="cuda")
    _capi.call("bee_b200_transpose_2d", 4, src.data_ptr() + 4, dst.data_ptr() + 4, rows, cols, stream(torch))
    torch.cuda.synchronize()
    assert np.array_equal(dst[1:].cpu().numpy(), a.reshape(rows, cols).T.reshape(-1))


def run_view(torch, dt, flat, offset, shape, strides):
    from bee_b200 import _capi
    npdt = DTYPES[dt]
    es = np.dtype(npdt).itemsize
    src = to_dev(torch, flat)
    n = int(np.prod(shape)) if len(shape) else 1
    dst = torch.zeros(max(n * es, 1), dtype=torch.uint8, device="cuda")
    nd = len(shape)
    sh = (ctypes.c_int64 * max(nd, 1))(*shape)
    st = (ctypes.c_int64 * max(nd, 1))(*strides)
    _capi.call("bee_b200_strided_copy", dt, src.data_ptr() + offset * es, nd, sh, st, dst.data_ptr(), stream(torch))
    torch.cuda.synchronize()
    return dst.cpu().numpy()[: n * es].view(npdt)


VIEWS = [
    # (base shape, offset, view shape, view strides)  — strides in elements
    ((2, 3, 4), 0, (4, 2, 3), (1, 12, 4)),                   # permute (2, 0, 1)
    ((32, 256, 128), 0, (32, 128, 256), (32768, 1, 128)),   # K^T of [heads, seq, d]
    ((4, 64, 8, 128), 64, (4, 64, 8, 64), (65536, 1024, 128, 1)),  # second half of every head (RoPE)
    ((4, 64, 8, 128), 0, (4, 64, 8, 64), (65536, 1024, 128, 1)),   # first half
    ((100, 37), 0, (100, 19), (37, 2)),                      # step-2 slice of the inner dim
    ((8, 1, 16), 0, (8, 5, 16), (16, 0, 1)),                 # broadcast (stride 0) view
    ((6, 10), 13, (3, 4), (20, 1)),                          # offset rows, inner run of 4
    ((300, 70), 0, (70, 300), (1, 70)),                      # plain 2-D transpose, ragged tiles
    ((5, 7, 9), 0, (9, 5, 7), (1, 63, 9)),                   # 3-D permute (2, 0, 1), gather path
    ((10,), 3, (), ()),                                      # 0-d view
    ((64,), 0, (64,), (1,)),                                 # already contiguous
]


@pytest.mark.parametrize("dt", [1, 4, 8, 3])
@pytest.mark.parametrize("view", VIEWS, ids=[f"v{i}" for i in range(len(VIEWS))])
def test_strided_copy(cuda, dt, view):
    base, offset, shape, strides = view
    rng = np.random.default_rng(len(shape) * 31 + offset + dt)
    flat = rand_bits(rng, int(np.prod(base)), DTYPES[dt])
    got = run_view(cuda, dt, flat, offset, shape, strides)
    want = Oracle.strided_gather(flat, offset, shape, strides).reshape(-1)
    assert np.array_equal(got, want)


def test_strided_copy_empty_and_errors(cuda):
    from bee_b200 import _capi
    torch = cuda
    sh = (ctypes.c_int64 * 2)(0, 5)
    st = (ctypes.c_int64 * 2)(5, 1)
    _capi.call("bee_b200_strided_copy", 4, None, 2, sh, st, None, stream(torch))  # zero elements: no-op
    sh9 = (ctypes.c_int64 * 9)(*([1] * 9))
    with pytest.raises(_capi.BeeError, match="ndim"):
        _capi.call("bee_b200_strided_copy", 4, 16, 9, sh9, sh9, 16, stream(torch))
    with pytest.raises(_capi.BeeError, match="dtype"):
        _capi.call("bee_b200_transpose_2d", 42, 16, 16, 4, 4, stream(torch))
