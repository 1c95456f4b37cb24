"""Partitioning of the Bee::Tensor path over the GPUs of one box.

One process per GPU; every rank calls the same kernels on its own shard, and
NCCL (through torch.distributed) carries the only exchange steps:

* row-wise ops (elementwise, cast, row reduce, softmax, RMSNorm, RoPE) shard by
  rows and need no collective;
* the global integer sum exchanges one partial per rank inside the reduce kernel
  (PeerReduce: the last block stores its partial into every rank's CUDA IPC
  receive array over NVLink and folds the world partials in rank order; integer
  addition wraps identically in any order, so the result is bit-exact);
* GEMM shards by output columns (no collective) or by K (split-K, SplitKGemm:
  the GEMM epilogue stores fp32 partial tiles straight into the owning GPU's
  receive buffer over NVLink, the owner sums and casts its tiles and writes
  them into every GPU's C; NCCL only supplies the two stream-ordered
  cross-GPU barriers);
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


def _exchange_handles(handle: bytes, world: int, group, device):
    """All-gathers one IPC handle (bytes) per rank over the process group."""
    import torch
    import torch.distributed as dist
    mine = torch.tensor(list(handle), dtype=torch.uint8, device=device)
    if world == 1:
        return [handle]
    allh = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allh, mine, group=group)
    return [bytes(h.cpu().tolist()) for h in allh]


class PeerReduce:
    """Global reduce over the ranks of one box in one kernel launch
    (bee_b200_reduce_global_allranks): every rank's dst receives the reduction
    of all ranks' inputs, folded in rank order.  Set-up allocates this rank's
    IPC receive array (one 8-byte slot per rank, zeroed), all-gathers the
    handles and opens the peers' arrays; each call uses a fresh tag."""

    def __init__(self, device, group=None, wait_ns: int = 2_000_000_000):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _capi
        self._capi = _capi
        self.device = torch.device(device)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("PeerReduce supports at most 8 GPUs")
        self.group, self.wait_ns, self.tag = group, int(wait_ns), 0
        self._own, self._opened = [], []
        buf = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _capi.call("bee_b200_ipc_alloc", ctypes.byref(buf), 256)
            self._own.append(buf.value)
            _capi.call("bee_b200_memset", buf, 0, 256, None)
            _capi.call("bee_b200_stream_synchronize", None)
            h = (ctypes.c_ubyte * 64)()
            _capi.call("bee_b200_ipc_handle", buf, ctypes.byref(h))
            ptrs = []
            for r, hb in enumerate(_exchange_handles(bytes(h), self.world, group, self.device)):
                if r == self.rank:
                    ptrs.append(buf.value)
                    continue
                out = ctypes.c_void_p()
                _capi.call("bee_b200_ipc_open", ctypes.byref((ctypes.c_ubyte * 64).from_buffer_copy(hb)),
                           ctypes.byref(out))
                self._opened.append(out.value)
                ptrs.append(out.value)
            self._slots = (ctypes.c_void_p * self.world)(*ptrs)
            torch.cuda.synchronize(self.device)

    def __call__(self, op: int, dt: int, src_ptr: int, n: int, dst_ptr: int, stream_ptr):
        self.tag = self.tag % 0xFFFFFFFF + 1  # 1 .. 2^32 - 1: never the zero of a fresh slot
        self._capi.call("bee_b200_reduce_global_allranks", op, dt, src_ptr, n, dst_ptr, self._slots, self.world,
                        self.rank, self.tag, self.wait_ns, stream_ptr)

    def close(self):
        import torch
        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)  # no peer still stores into our array
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                self._capi.call("bee_b200_ipc_close", ptr)
            for ptr in self._own:
                self._capi.call("bee_b200_ipc_free", ptr)
        self._opened, self._own = [], []


class SplitKGemm:
    """C = A . B with K sharded over the ranks of one box, fused with its
    reduction over NVLink peer memory (one process per GPU, NCCL process group).

    Rank r passes A[:, K_r] (a column block of the row-major [M, K] A: base
    pointer and row stride `lda`) and B[K_r, :] ([K_r, N] row-major); every rank
    receives the full bf16 C = sum_r A[:, K_r] . B[K_r, :] in its own `c`.

    Set-up (once per shape): each rank allocates an IPC-shareable receive buffer
    (bee_b200_splitk_recv_bytes) and its C, exports both handles, all-gathers
    them and opens the peers' buffers.  Per call, on the caller's stream:
    scatter GEMM -> barrier -> owner reduce + C broadcast -> barrier.  The
    barriers are one-element NCCL all-reduces, ordered on the same stream.
    """

    def __init__(self, M: int, N: int, device, group=None):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _capi
        self._capi = _capi
        self.M, self.N, self.group = M, N, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("split-K GEMM supports at most 8 GPUs")
        self.device = torch.device(device)
        self._recv_bytes = int(_capi.lib().bee_b200_splitk_recv_bytes(M, N, self.world))
        self._own = []    # (pointer) buffers this rank allocated
        self._opened = []  # peer mappings opened in this process
        recv = ctypes.c_void_p()
        cbuf = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _capi.call("bee_b200_ipc_alloc", ctypes.byref(recv), self._recv_bytes)
            self._own.append(recv.value)
            _capi.call("bee_b200_ipc_alloc", ctypes.byref(cbuf), max(M * N * 2, 16))
            self._own.append(cbuf.value)
            handles = (ctypes.c_ubyte * 128)()
            _capi.call("bee_b200_ipc_handle", ctypes.c_void_p(recv.value), ctypes.byref(handles, 0))
            _capi.call("bee_b200_ipc_handle", ctypes.c_void_p(cbuf.value), ctypes.byref(handles, 64))
            mine = torch.tensor(list(bytes(handles)), dtype=torch.uint8, device=self.device)
            if self.world > 1:
                allh = [torch.empty_like(mine) for _ in range(self.world)]
                dist.all_gather(allh, mine, group=group)
                allh = [bytes(h.cpu().tolist()) for h in allh]
            else:
                allh = [bytes(handles)]
            self.recv_local = recv.value
            self.c_local = cbuf.value
            recv_peers, c_peers = [], []
            for r, h in enumerate(allh):
                if r == self.rank:
                    recv_peers.append(recv.value)
                    c_peers.append(cbuf.value)
                    continue
                ptrs = []
                for off in (0, 64):
                    hb = (ctypes.c_ubyte * 64).from_buffer_copy(h[off:off + 64])
                    out = ctypes.c_void_p()
                    _capi.call("bee_b200_ipc_open", ctypes.byref(hb), ctypes.byref(out))
                    self._opened.append(out.value)
                    ptrs.append(out.value)
                recv_peers.append(ptrs[0])
                c_peers.append(ptrs[1])
            self._recv_peers = (ctypes.c_void_p * self.world)(*recv_peers)
            self._c_peers = (ctypes.c_void_p * self.world)(*c_peers)
            self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
            torch.cuda.synchronize(self.device)
        # C as a tensor view of the IPC buffer (the library owns the memory)
        self.c = _wrap_bf16(self.c_local, M, N, self.device)

    def barrier(self):
        """Stream-ordered cross-GPU barrier on the current stream."""
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(self._flag, group=self.group)

    def __call__(self, a_ptr: int, lda: int, b_ptr: int, k_local: int, stream_ptr: int):
        """Launches the scatter GEMM, the barrier, the owner reduce and the
        closing barrier on the current torch stream (whose handle is stream_ptr)."""
        _capi = self._capi
        _capi.call("bee_b200_gemm_splitk_scatter", a_ptr, lda, b_ptr, self.M, k_local, self.N, self._recv_peers,
                   self.world, self.rank, stream_ptr)
        self.barrier()
        _capi.call("bee_b200_gemm_splitk_reduce", self.recv_local, self._c_peers, self.M, self.N, self.world,
                   self.rank, stream_ptr)
        self.barrier()
        return self.c

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (after a device sync
        and a barrier, so no rank still writes into them)."""
        import torch
        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        self.barrier()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                self._capi.call("bee_b200_ipc_close", ptr)
            for ptr in self._own:
                self._capi.call("bee_b200_ipc_free", ptr)
        self._opened, self._own = [], []


def _wrap_bf16(ptr: int, M: int, N: int, device):
    """A [M, N] bf16 torch view of device memory at `ptr` (not owned)."""
    import torch

    class _Iface:
        __cuda_array_interface__ = {"shape": (M, N), "typestr": "<i2", "data": (ptr, False), "version": 3,
                                    "strides": None}
    return torch.as_tensor(_Iface(), device=device).view(torch.bfloat16)
