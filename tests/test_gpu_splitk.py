"""GPU parity of the split-K GEMM fused with its reduction
(bee_b200_gemm_splitk_scatter / bee_b200_gemm_splitk_reduce).

The reference has no multi-GPU GEMM; its single-GPU product
(Bee/CUDA/Ops/Matmul.cu, bf16 in, fp32 accumulate) is the oracle.  Two checks:

* bit-exact: C must equal bf16_rne(0 + P_0 + P_1 + ... + P_{w-1}) where P_r is
  rank r's fp32 partial product computed by the single-GPU bee_b200_bmm (the
  same tensor-core instruction sequence), summed in rank order;
* oracle: C within the bf16 output tolerance of the float64-accumulated
  product (1e-2 of the |A||B| condition).

World sizes 1-8 are emulated on one GPU: every "rank" launches its scatter on
the same stream (no kernel waits on another), then every owner its reduce.  The
real multi-process path (CUDA IPC, NCCL barriers) runs in tests/_splitk_worker.py
when two GPUs are present.
"""
import os
import subprocess
import sys
from pathlib import Path

import ctypes
import numpy as np
import pytest

from tests._tol import assert_dot_close
from oracle.oracle import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def status_word():
    from bee_b200 import _capi
    code = ctypes.c_int(-1)
    _capi.call("bee_b200_device_status", ctypes.byref(code))
    return code.value


def k_slices(k, world):
    """K shards in multiples of 8 (16-byte aligned column blocks of A)."""
    from bee_b200.shard import shard_range
    return [tuple(8 * x for x in shard_range(k // 8, world, r)) for r in range(world)]


def emulated_splitk(torch, a, b, world):
    """Runs the fused split-K for `world` emulated ranks on one GPU; returns
    every rank's C (bf16 as int16) and every rank's fp32 partial from bmm."""
    from bee_b200 import _capi
    m, k = a.shape
    n = b.shape[1]
    st = torch.cuda.current_stream().cuda_stream
    recv_bytes = _capi.lib().bee_b200_splitk_recv_bytes(m, n, world)
    recv = [torch.full((recv_bytes // 4,), float("nan"), dtype=torch.float32, device="cuda") for _ in range(world)]
    cs = [torch.full((m, n), -1, dtype=torch.int16, device="cuda") for _ in range(world)]
    recv_ptrs = (ctypes.c_void_p * world)(*[t.data_ptr() for t in recv])
    c_ptrs = (ctypes.c_void_p * world)(*[t.data_ptr() for t in cs])
    slices = k_slices(k, world)
    for r, (lo, hi) in enumerate(slices):
        _capi.call("bee_b200_gemm_splitk_scatter", a.data_ptr() + 2 * lo, k, b[lo:hi].data_ptr(), m, hi - lo, n,
                   recv_ptrs, world, r, st)
    for r in range(world):
        _capi.call("bee_b200_gemm_splitk_reduce", recv[r].data_ptr(), c_ptrs, m, n, world, r, st)
    parts = []
    for lo, hi in slices:
        ak = a[:, lo:hi].contiguous()
        bk = b[lo:hi].contiguous()
        p = torch.empty(m, n, dtype=torch.float32, device="cuda")
        _capi.call("bee_b200_bmm", _capi.BF16, _capi.F32, ak.data_ptr(), bk.data_ptr(), p.data_ptr(), 1, m, hi - lo,
                   n, 0, 1.0, st)
        parts.append(p)
    torch.cuda.synchronize()
    assert status_word() == 0, "a tensor-core pipeline wait gave up"
    return cs, parts


def expected_bits(torch, parts):
    acc = torch.zeros_like(parts[0])
    for p in parts:
        acc += p
    return acc.to(torch.bfloat16).view(torch.int16)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("m,k,n", [(520, 1024, 776), (256, 512, 256), (1000, 2056, 264)])
def test_splitk_bit_exact(cuda, world, m, k, n):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(1000 * world + m)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16).view(torch.int16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16).view(torch.int16)
    cs, parts = emulated_splitk(torch, a, b, world)
    want = expected_bits(torch, parts)
    for r, c in enumerate(cs):
        mismatch = int((c != want).sum())
        assert mismatch == 0, f"rank {r}: {mismatch} of {m * n} entries differ from the rank-ordered fp32 sum"


@pytest.mark.parametrize("world", [2, 8])
def test_splitk_vs_oracle(cuda, oracle, world):
    torch = cuda
    rng = np.random.default_rng(77 + world)
    m, k, n = 300, 1536, 520
    a_bits = f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    b_bits = f32_to_bf16_bits(rng.standard_normal((k, n)).astype(np.float32))
    a = torch.from_numpy(a_bits.view(np.int16)).cuda()
    b = torch.from_numpy(b_bits.view(np.int16)).cuda()
    cs, _ = emulated_splitk(torch, a, b, world)
    ref = oracle.bmm_bf16(a_bits, b_bits)[0]
    got = bf16_bits_to_f32(cs[0].cpu().numpy().view(np.uint16))
    assert_dot_close(got, ref, bf16_bits_to_f32(a_bits), bf16_bits_to_f32(b_bits), 1e-2, "split-K bf16")


def test_splitk_rejects_bad_arguments(cuda):
    from bee_b200 import _capi
    torch = cuda
    a = torch.zeros(256, 256, dtype=torch.int16, device="cuda")
    buf = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    ptrs = (ctypes.c_void_p * 1)(buf.data_ptr())
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(_capi.BeeError, match="misaligned|multiples of 8"):
        _capi.call("bee_b200_gemm_splitk_scatter", a.data_ptr() + 2, 256, a.data_ptr(), 256, 248, 256, ptrs, 1, 0, st)
    with pytest.raises(_capi.BeeError, match="out of range"):
        _capi.call("bee_b200_gemm_splitk_reduce", buf.data_ptr(), ptrs, 256, 256, 1, 1, st)


def test_splitk_two_processes():
    """The real path: two processes on two GPUs, CUDA IPC buffers, NCCL barriers."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_DEBUG="WARN", NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531",
           str(ROOT / "tests" / "_splitk_worker.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count("SPLITK_OK") == 2, res.stdout[-3000:]
