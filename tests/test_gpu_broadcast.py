"""GPU parity of the broadcasting / strided binary op (bee_b200_ew_binary_strided)
against the oracle's binary op under numpy broadcasting (pinned to the
reference's CPU broadcast in tests/test_oracle_layout.py).  Bit-exact for
every dtype: the kernel computes in the same types as bee_b200_ew_binary."""
import ctypes

import numpy as np
import pytest

from oracle.oracle import Oracle, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu

NP = {1: np.uint8, 2: np.int32, 3: np.int64, 4: np.float32, 5: np.float64, 8: np.uint16}


def rand(rng, shape, dt, divisor=False):
    if dt == 1:
        return rng.integers(1 if divisor else 0, 256, size=shape, dtype=np.uint8)
    if dt in (2, 3):
        x = rng.integers(-1000, 1000, size=shape).astype(NP[dt])
        if divisor:
            x[x == 0] = 7
        return x
    x = rng.standard_normal(shape)
    if divisor:
        x = x + np.where(x >= 0, 0.5, -0.5)
    if dt == 8:
        return f32_to_bf16_bits(x.astype(np.float32))
    return x.astype(NP[dt])


def oracle_binary(op, dt, a, b):
    if dt == 8:
        return f32_to_bf16_bits(Oracle.binary(op, bf16_bits_to_f32(a), bf16_bits_to_f32(b)))
    return Oracle.binary(op, a, b)


def run(torch, op, dt, shape, a_buf, a_off, a_str, b_buf, b_off, b_str):
    from bee_b200 import _capi
    es = np.dtype(NP[dt]).itemsize
    da = torch.from_numpy(np.ascontiguousarray(a_buf).reshape(-1).view(np.uint8).copy()).cuda()
    db = torch.from_numpy(np.ascontiguousarray(b_buf).reshape(-1).view(np.uint8).copy()).cuda()
    n = int(np.prod(shape)) if len(shape) else 1
    out = torch.zeros(max(n * es, 1), dtype=torch.uint8, device="cuda")
    nd = len(shape)
    arr = lambda v: (ctypes.c_int64 * max(nd, 1))(*v)
    _capi.call("bee_b200_ew_binary_strided", op, dt, nd, arr(shape), da.data_ptr() + a_off * es, arr(a_str),
               db.data_ptr() + b_off * es, arr(b_str), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy()[: n * es].view(NP[dt]).reshape(shape)


def bcast_strides(shape_op, shape_out):
    """Contiguous strides of an operand of shape_op broadcast to shape_out (0 on broadcast dims)."""
    st = np.cumprod((list(shape_op[1:]) + [1])[::-1])[::-1] if shape_op else []
    return [0 if so == 1 and n != 1 else int(s) for so, n, s in zip(shape_op, shape_out, st)]


CASES = [
    ((512, 300), (512, 1)),      # x - rowmax(x) (keepdim), softmax composition
    ((512, 300), (1, 300)),      # x * w, RMSNorm weight
    ((4, 1, 7), (1, 5, 7)),      # both operands broadcast
    ((3, 4, 5), (3, 4, 5)),      # same shape (contiguous fast path)
    ((64, 128), (1, 1)),         # scalar operand
    ((2, 3, 1, 33), (2, 1, 6, 1)),
    ((1000,), (1,)),
    ((257, 129), (257, 1)),      # odd row length: partial vectors at every row end
]


@pytest.mark.parametrize("dt", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("ashape,bshape", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_broadcast_binary(cuda, dt, op, ashape, bshape):
    rng = np.random.default_rng(hash((dt, op, ashape, bshape)) % (2 ** 32))
    a = rand(rng, ashape, dt)
    b = rand(rng, bshape, dt, divisor=(op == 3))
    shape = np.broadcast_shapes(ashape, bshape)
    got = run(cuda, op, dt, shape, a, 0, bcast_strides(ashape, shape), b, 0, bcast_strides(bshape, shape))
    want = oracle_binary(op, dt, a, b)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dt", [4, 8])
def test_strided_operands(cuda, dt):
    """Non-contiguous operands: a transposed view and a step-2 slice with an offset."""
    rng = np.random.default_rng(5)
    base_a = rand(rng, (96, 80), dt)          # a = base_a^T, shape (80, 96)
    base_b = rand(rng, (80, 200), dt)         # b = base_b[:, 3:195:2], shape (80, 96)
    shape = (80, 96)
    got = run(cuda, 0, dt, shape, base_a, 0, (1, 80), base_b, 3, (200, 2))
    a_view = Oracle.strided_gather(base_a.reshape(-1), 0, shape, (1, 80))
    b_view = Oracle.strided_gather(base_b.reshape(-1), 3, shape, (200, 2))
    assert np.array_equal(got, oracle_binary(0, dt, a_view, b_view))


def test_zero_dim_and_empty(cuda):
    from bee_b200 import _capi
    a = np.array([2.5], np.float32)
    b = np.array([4.0], np.float32)
    got = run(cuda, 2, 4, (), a, 0, (), b, 0, ())
    assert float(got) == 10.0
    sh = (ctypes.c_int64 * 2)(0, 3)
    _capi.call("bee_b200_ew_binary_strided", 0, 4, 2, sh, None, sh, None, sh, None, None)
    with pytest.raises(_capi.BeeError, match="ndim"):
        _capi.call("bee_b200_ew_binary_strided", 0, 4, 9, sh, 16, sh, 16, sh, 16, None)
