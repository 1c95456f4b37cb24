"""GPU checks of the global reduce across GPUs (bee_b200_reduce_global_allranks)
that run on one GPU: world 1 (the rank's own slot only) against the oracle and
the single-GPU reduce, and the failure path — a peer that never delivers its
partial — made with a slot that nothing writes (the kernel's wait runs out after
a short limit, records a status code and leaves the local partial).  The
two-process path runs in tests/_splitk_worker.py."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def status_word():
    from bee_b200 import _capi
    code = ctypes.c_int(-1)
    _capi.call("bee_b200_device_status", ctypes.byref(code))
    return code.value


def allranks(torch, op, dt, x, slots, world, rank, tag, wait_ns=2_000_000_000):
    from bee_b200 import _capi
    out = torch.zeros(1, dtype=x.dtype, device="cuda")
    arr = (ctypes.c_void_p * world)(*[s.data_ptr() for s in slots])
    _capi.call("bee_b200_reduce_global_allranks", op, dt, x.data_ptr(), x.numel(), out.data_ptr(), arr, world, rank,
               tag, wait_ns, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out


def single(torch, op, dt, x):
    from bee_b200 import _capi
    out = torch.zeros(1, dtype=x.dtype, device="cuda")
    _capi.call("bee_b200_reduce_global", op, dt, x.data_ptr(), out.data_ptr(), x.numel(),
               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("n", [1, 257, (1 << 20) + 3, 8192 * 8192])
def test_world1_matches_single_gpu_reduce(cuda, oracle, n):
    from bee_b200 import _capi
    torch = cuda
    rng = np.random.default_rng(n)
    xi = rng.integers(-1000, 1001, n).astype(np.int32)
    xf = rng.standard_normal(n).astype(np.float32)
    di, df = torch.from_numpy(xi).cuda(), torch.from_numpy(xf).cuda()
    slot = torch.zeros(16, dtype=torch.int64, device="cuda")
    tag = 1
    for op in (_capi.SUM, _capi.MIN, _capi.MAX):
        got = allranks(torch, op, _capi.I32, di, [slot], 1, 0, tag)
        tag += 1
        assert int(got.item()) == int(single(torch, op, _capi.I32, di).item())
        gotf = allranks(torch, op, _capi.F32, df, [slot], 1, 0, tag)
        tag += 1
        assert gotf.view(torch.int32).item() == single(torch, op, _capi.F32, df).view(torch.int32).item()
    assert int(allranks(torch, _capi.SUM, _capi.I32, di, [slot], 1, 0, tag).item()) == oracle.reduce_global_i32(0, xi)
    assert status_word() == 0


def test_missing_peer_times_out_with_status(cuda):
    """Rank 0 of a world of 2 whose peer never stores: the wait gives up after
    20 ms, the status word names the missing slot (40 + 1), dst holds the local
    partial, and the next call works."""
    from bee_b200 import _capi
    torch = cuda
    x = torch.arange(1000, dtype=torch.int32, device="cuda")
    own = torch.zeros(16, dtype=torch.int64, device="cuda")
    other = torch.zeros(16, dtype=torch.int64, device="cuda")
    got = allranks(torch, _capi.SUM, _capi.I32, x, [own, other], 2, 0, tag=1, wait_ns=20_000_000)
    assert int(got.item()) == 999 * 1000 // 2
    assert status_word() == 41
    assert status_word() == 0  # read-and-clear
    ok = allranks(torch, _capi.SUM, _capi.I32, x, [own], 1, 0, tag=2)
    assert int(ok.item()) == 999 * 1000 // 2 and status_word() == 0


def test_rejects_bad_arguments(cuda):
    from bee_b200 import _capi
    torch = cuda
    x = torch.zeros(8, dtype=torch.int32, device="cuda")
    slot = torch.zeros(16, dtype=torch.int64, device="cuda")
    with pytest.raises(_capi.BeeError, match="tag 0"):
        allranks(torch, _capi.SUM, _capi.I32, x, [slot], 1, 0, tag=0)
    with pytest.raises(_capi.BeeError, match="I32 or F32"):
        allranks(torch, _capi.SUM, _capi.I64, x, [slot], 1, 0, tag=1)
    with pytest.raises(_capi.BeeError, match="out of range"):
        allranks(torch, _capi.SUM, _capi.I32, x, [slot], 1, 1, tag=1)
