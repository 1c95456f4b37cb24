"""CPU pins of the integer-mean oracle against the reference's own CPU mean
(compiled from its sources), global and per axis, I32 and I64."""
import numpy as np
import pytest

from oracle.oracle import Oracle


@pytest.mark.parametrize("dtype", [np.int32, np.int64])
@pytest.mark.parametrize("shape", [(1, 1, 1), (1, 4099, 1), (5, 300, 1), (6, 50, 33), (2, 7, 16)])
def test_mean_int_oracle_matches_reference(reference, dtype, shape):
    rng = np.random.default_rng(sum(shape))
    x = rng.integers(-1000, 1001, size=shape).astype(dtype)
    if dtype == np.int64:
        x = x * np.int64(1 << 30)
    got_axis, _ = reference.mean_int(x)
    assert np.array_equal(Oracle.mean_int(x, axis=1), got_axis)
    got_all, _ = reference.mean_int(x, global_mean=True)
    assert Oracle.mean_int(x) == got_all


def test_mean_int_known_answer():
    """mean of 1..10 = 5.5; of [-3, 4] = 0.5 (F64)."""
    assert Oracle.mean_int(np.arange(1, 11, dtype=np.int32)) == 5.5
    assert Oracle.mean_int(np.array([[-3, 4]], np.int64), axis=1)[0] == 0.5
