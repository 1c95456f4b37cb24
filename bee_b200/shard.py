"""Partitioning of the Bee::Tensor path over the GPUs of one box.

One process per GPU; every rank calls the same kernels on its own shard, and
NCCL (through torch.distributed) carries the only exchange steps:

* row-wise ops (elementwise, cast, row reduce, softmax, RMSNorm, RoPE) shard by
  rows and need no collective;
* the global integer sum all-reduces one partial per rank (integer addition
  wraps identically in any order, so the result is bit-exact);
* GEMM shards by output columns (no collective) or by K (split-K: fp32 partial
  products summed by an all-reduce, then cast);
* attention shards by heads (no collective).
"""
from __future__ import annotations


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced [lo, hi) slice of `total` units for `rank`: the first
    total % world ranks get one extra unit."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if total < 0:
        raise ValueError("negative extent")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def allreduce_sum_(tensor, group=None):
    """In-place sum of `tensor` over the ranks of `group` (NCCL on GPUs, gloo on CPU)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=group)
    return tensor


def allgather_rows(local, group=None):
    """Concatenates every rank's row shard along dim 0 (equal shard sizes)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return local
    parts = [torch.empty_like(local) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, 0)
