"""The N>1 path on CPU: world_size-2 gloo process groups run the sharding and
combine steps of bee_b200.shard with the oracle as the per-rank compute, and a
rank that never joins makes the others fail with an error instead of hanging."""
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bee_b200.shard import allgather_rows, allreduce_sum_, shard_range


def test_shard_range_partitions_exactly():
    for total in [0, 1, 7, 8192, 32768, 10001]:
        for world in [1, 2, 3, 4, 8]:
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn, errq):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        fn(rank, world)
        dist.destroy_process_group()
        errq.put((rank, None))
    except Exception:
        errq.put((rank, traceback.format_exc()))


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, errq)) for r in range(world)]
    for p in procs:
        p.start()
    results = [errq.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    errs = [e for _, e in results if e]
    assert not errs, "\n".join(errs)


def _int_sum_rank(rank, world):
    from oracle.oracle import Oracle
    orc = Oracle()
    x = np.random.default_rng(5).integers(-1000, 1001, (1000, 333)).astype(np.int32)
    lo, hi = shard_range(x.shape[0], world, rank)
    part = torch.tensor([orc.reduce_global_i32(0, x[lo:hi])], dtype=torch.int32)
    allreduce_sum_(part)
    assert int(part.item()) == orc.reduce_global_i32(0, x)


def _split_k_rank(rank, world):
    from oracle.oracle import Oracle
    orc = Oracle()
    rng = np.random.default_rng(6)
    a = rng.uniform(-1, 1, (48, 256)).astype(np.float32)
    b = rng.uniform(-1, 1, (256, 40)).astype(np.float32)
    lo, hi = shard_range(a.shape[1], world, rank)
    part = torch.from_numpy(orc.matmul_f32(np.ascontiguousarray(a[:, lo:hi]), np.ascontiguousarray(b[lo:hi])))
    allreduce_sum_(part)
    full = orc.matmul_f32(a, b)
    scale = np.abs(a) @ np.abs(b)
    assert np.max(np.abs(part.numpy() - full) / scale) < 1e-4


def _row_gather_rank(rank, world):
    from oracle.oracle import Oracle
    orc = Oracle()
    x = np.random.default_rng(7).standard_normal((64, 300)).astype(np.float32)
    lo, hi = shard_range(64, world, rank)
    local = torch.from_numpy(orc.softmax_f32(x[lo:hi]))
    full = allgather_rows(local)
    np.testing.assert_array_equal(full.numpy(), orc.softmax_f32(x))


def _departed_worker(rank, world, port, q):
    """Step 1 runs on both ranks; rank 1 then leaves between steps (exits
    without tearing the group down); rank 0's step-2 collective must raise,
    within the group's timeout, rather than hang or complete."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        t = torch.ones(1)
        dist.all_reduce(t)
        if rank == 1:
            q.put((1, "left after step 1", float(t.item()), 0.0))
            q.close()
            q.join_thread()  # the message is sent before the process leaves
            os._exit(0)
        t0 = time.monotonic()
        try:
            dist.all_reduce(torch.ones(1))
            q.put((0, "completed", float(t.item()), time.monotonic() - t0))
        except Exception as e:  # the expected outcome
            q.put((0, f"raised {type(e).__name__}", float(t.item()), time.monotonic() - t0))
    except Exception:
        q.put((rank, "failed before step 2: " + traceback.format_exc(), 0.0, 0.0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_int32_sum_over_two_ranks():
    _run(_int_sum_rank)


def test_split_k_gemm_over_two_ranks():
    _run(_split_k_rank)


def test_row_sharded_softmax_gather_over_two_ranks():
    _run(_row_gather_rank)


def test_departed_rank_fails_the_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_departed_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, outcome, step1, elapsed = q.get(timeout=120)
        results[rank] = (outcome, step1, elapsed)
    for p in procs:
        p.join(timeout=60)
    assert results[1][:2] == ("left after step 1", 2.0), results
    outcome, step1, elapsed = results[0]
    assert step1 == 2.0, results  # step 1 completed on rank 0 as well
    assert outcome.startswith("raised "), f"rank 0's collective after rank 1 left: {outcome}"
    assert elapsed < 60.0, f"rank 0 learned of the departure only after {elapsed:.1f} s"
