"""One rank of the two-process checks of the multi-GPU paths (launched by
tests/test_gpu_splitk.py under torch.distributed.run, one process per GPU):
the split-K GEMM and the cross-GPU global reduce (PeerReduce).

Every rank builds the same A [M, K] and B [K, N] (same seed), multiplies its
K shard through SplitKGemm (peer stores over NVLink, NCCL barriers), and checks
its full C bit for bit against bf16_rne(0 + P_0 + P_1) with P_r the fp32
partials of the single-GPU bee_b200_bmm, gathered with NCCL.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def main():
    import torch
    import torch.distributed as dist
    from bee_b200 import _capi
    from bee_b200.shard import PeerReduce, SplitKGemm, shard_range

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for (m, k, n) in [(520, 1024, 776), (2048, 4096, 2048)]:
            g = torch.Generator(device=dev).manual_seed(5 + m)
            a = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            b = torch.randn(k, n, device=dev, generator=g).to(torch.bfloat16)
            lo, hi = (8 * x for x in shard_range(k // 8, world, rank))
            gemm = SplitKGemm(m, n, dev)
            for _ in range(3):  # repeated calls reuse the receive buffers
                c = gemm(a.data_ptr() + 2 * lo, k, b[lo:hi].data_ptr(), hi - lo, stream.cuda_stream)
            ak, bk = a[:, lo:hi].contiguous(), b[lo:hi].contiguous()
            part = torch.empty(m, n, dtype=torch.float32, device=dev)
            _capi.call("bee_b200_bmm", _capi.BF16, _capi.F32, ak.data_ptr(), bk.data_ptr(), part.data_ptr(), 1, m,
                       hi - lo, n, 0, 1.0, stream.cuda_stream)
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            acc = torch.zeros_like(part)
            for p in parts:
                acc += p
            want = acc.to(torch.bfloat16)
            got = c.clone()
            stream.synchronize()
            bad = int((got.view(torch.int16) != want.view(torch.int16)).sum())
            gemm.close()
            if bad:
                print(f"rank {rank}: {bad} of {m * n} entries differ ({m}x{k}x{n})", flush=True)
                dist.destroy_process_group()
                sys.exit(1)
        # cross-GPU int32 sum: every call (both tag banks) equals the NCCL sum of the partials
        pr = PeerReduce(dev)
        for call in range(5):
            g = torch.Generator(device=dev).manual_seed(100 * call + rank)
            x = torch.randint(-1000, 1001, ((1 << 20) + 7 * call,), device=dev, generator=g, dtype=torch.int32)
            out = torch.zeros(1, dtype=torch.int32, device=dev)
            pr(_capi.SUM, _capi.I32, x.data_ptr(), x.numel(), out.data_ptr(), stream.cuda_stream)
            part = torch.zeros(1, dtype=torch.int32, device=dev)
            _capi.call("bee_b200_reduce_global", _capi.SUM, _capi.I32, x.data_ptr(), part.data_ptr(), x.numel(),
                       stream.cuda_stream)
            dist.all_reduce(part)
            stream.synchronize()
            if int(out.item()) != int(part.item()):
                print(f"rank {rank}: peer reduce {int(out.item())} != {int(part.item())} (call {call})", flush=True)
                dist.destroy_process_group()
                sys.exit(1)
        pr.close()
    dist.destroy_process_group()
    print(f"SPLITK_OK rank {rank}", flush=True)


if __name__ == "__main__":
    main()
