"""CPU pins of the layout oracle (strided gather / transpose) against the
reference's known answers and against the reference's own CPU
materialisation of views (permute + slice + contiguous, compiled from its
sources)."""
import numpy as np
import pytest

from oracle.oracle import Oracle


def test_contiguous_data_order_kat():
    """Tests/Tensor/ViewTests.cpp:152-186: transpose of [[0,1,2],[3,4,5]] -> {0,3,1,4,2,5}."""
    flat = np.arange(6, dtype=np.float32)
    out = Oracle.strided_gather(flat, 0, (3, 2), (1, 3))
    assert out.reshape(-1).tolist() == [0, 3, 1, 4, 2, 5]


def test_transpose_kats():
    """Tests/CUDA/TransposeTests.cu:79-110 (3x5 f64 i*0.5; 32x64 f32 ((i%17)-8)*0.25)."""
    a = np.arange(15, dtype=np.float64) * 0.5
    got = Oracle.strided_gather(a, 0, (5, 3), (1, 5))
    assert np.array_equal(got, a.reshape(3, 5).T)
    b = ((np.arange(32 * 64) % 17) - 8).astype(np.float32) * 0.25
    got = Oracle.strided_gather(b, 0, (64, 32), (1, 64))
    assert np.array_equal(got, b.reshape(32, 64).T)


@pytest.mark.parametrize("shape,perm,slices", [
    ((2, 3, 4), (2, 0, 1), None),
    ((4, 6, 8), (1, 2, 0), [None, (1, 7, 2), (0, 4, 1)]),
    ((3, 5, 7, 9), (0, 2, 1, 3), [None, None, None, (0, 9, 3)]),
    ((16, 8, 64), (0, 2, 1), None),
    ((2, 8, 4, 16), (0, 1, 2, 3), [None, None, None, (8, 16, 1)]),
])
def test_strided_gather_matches_reference(reference, shape, perm, slices):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(shape).astype(np.float32)
    want, _ = reference.view_copy_f32(x, perm, slices)
    # the same view by offset/shape/strides
    st = np.array(x.strides) // 4
    vshape = [shape[p] for p in perm]
    vstr = [int(st[p]) for p in perm]
    off = 0
    for d, sl in enumerate(slices or [None] * len(shape)):
        if sl is None:
            continue
        off += sl[0] * vstr[d]
        vshape[d] = len(range(*sl))
        vstr[d] *= sl[2]
    got = Oracle.strided_gather(x.reshape(-1), off, vshape, vstr)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("ashape,bshape", [((64, 48), (64, 1)), ((64, 48), (1, 48)), ((4, 1, 7), (1, 5, 7)),
                                           ((3, 4, 5), (3, 4, 5))])
def test_broadcast_binary_oracle_matches_reference(reference, op, ashape, bshape):
    """numpy broadcasting of the oracle's binary op equals the reference's CPU broadcast."""
    rng = np.random.default_rng(op * 11 + len(ashape))
    a = rng.standard_normal(ashape).astype(np.float32)
    b = (rng.standard_normal(bshape) + 3.0).astype(np.float32)
    want, _ = reference.binary_bcast_f32(op, a, b)
    got = Oracle.binary(op, a, b)
    assert got.shape == want.shape and np.array_equal(got, want)
