"""Benchmark of the Bee::Tensor hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload sweep]

Workload "sweep" (the headline): the memory-bound op sweep on row-major
[8192, 8192] tensors — fp32 add and mul of two N(0,1) tensors, fp32->bf16 cast,
row sum, row max, row softmax, and the bit-exact int32 full sum of a uniform
[-1000, 1000] tensor.  A step runs every op once over the GPU's shard; rows are
sharded over GPUs with 8192 rows per GPU (weak scaling: the global tensor is
[8192*N, 8192]); the only exchange is the int32 sum's: an NCCL all-reduce of
the per-GPU partials, or with --exchange peer the exchange inside the reduce
kernel over NVLink peer memory (bee_b200.shard.PeerReduce).  Each tensor is 256 MiB, larger than the 126 MB L2, so no L2 flush is
needed between ops or steps.  ``value`` is the algorithmic bytes moved by all
ranks per second (GB/s, 1e9).

``--impl reference`` times the reference's own CPU implementation of the same
ops (the Bee::Tensor CPU path compiled from the reference sources into
oracle/_ref, else the oracle port) on the host cores, rank 0 only.

``--only NAME`` (profiling) skips the sweep and runs one of the extra configs
alone (gemm_bf16_8192, rms_norm_rope_bf16, attention_bf16, gemm_f32_1024,
transpose_f32_8192, ...), printing {"only": NAME, "extra": {...}}; the ncu
captures of those kernels use it so that they run this file and nothing else.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, COLS = 8192, 8192
N_EL = ROWS * COLS
F32_BYTES = N_EL * 4
# algorithmic bytes per op over one 8192 x 8192 shard
OP_BYTES = {
    "add_f32": 3 * F32_BYTES,
    "mul_f32": 3 * F32_BYTES,
    "cast_f32_bf16": F32_BYTES + N_EL * 2,
    "row_sum_f32": F32_BYTES + ROWS * 4,
    "row_max_f32": F32_BYTES + ROWS * 4,
    "softmax_f32": 2 * F32_BYTES,
    "sum_i32": F32_BYTES + 4,
}
STEP_BYTES = sum(OP_BYTES.values())
# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of each
# sweep kernel, from one ncu capture of this bench's own command.  Writes still
# dirty in L2 when a kernel ends are not counted, hence slightly below the
# algorithmic bytes.
NCU_TRAFFIC = {
    "add_f32": 768_840_000, "mul_f32": 770_200_000, "cast_f32_bf16": 359_370_000,
    "row_sum_f32": 268_870_000, "row_max_f32": 268_560_000, "softmax_f32": 486_080_000, "sum_i32": 269_000_000,
}


SWEEP_OPS = ["add_f32", "mul_f32", "cast_f32_bf16", "row_sum_f32", "row_max_f32", "softmax_f32", "sum_i32"]


def sweep_config(world: int, peer_exchange: bool = False) -> dict:
    """The workload both arms report (the reference arm runs the same workload
    on the host cores)."""
    return {"workload": "memory-bound op sweep, [8192, 8192] fp32 + int32 per GPU, rows sharded "
                        "(8192 rows per GPU, global [8192*N, 8192])",
            "ops": SWEEP_OPS, "bytes_per_step_per_gpu": STEP_BYTES,
            "l2": "inputs larger than L2 (each tensor 256 MiB > 126 MB), no flush",
            "parallelism": (f"rows sharded over {world} GPUs; int32 partial sums combined "
                            + ("inside the reduce kernel over NVLink peer memory" if peer_exchange
                               else "by an NCCL all-reduce")) if world > 1 else "1 GPU"}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """Samples the SM clock (every period) and the clock-event (throttle) reasons
    (every `reasons_every` samples) through NVML while the timed region runs
    (nvidia-smi's 200 ms period is longer than the region).  One thread, in rank
    0's process: NVML queries stretch cross-GPU waits (NCCL's and ours) on the
    queried GPU, a sampler in every rank or in a separate process much more so
    than one thread in one rank, and the reasons query more than the clock one."""

    def __init__(self, bus_id: str, period_s: float = 0.002, enabled: bool = True, reasons_every: int = 10,
                 at_s=None):
        self.enabled = enabled
        self.bus_id = bus_id
        self.period = period_s
        self.at_s = at_s  # instead of periodic sampling: one sample per offset (seconds after entry)
        self.reasons_every = max(1, reasons_every)
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self.error = None

    def __enter__(self):
        if not self.enabled:
            self.error = "disabled (--no-clocks, or not rank 0)"
            return self
        try:
            import pynvml as nv
            nv.nvmlInit()
            self._nvml = nv
            self._h = nv.nvmlDeviceGetHandleByPciBusId(self.bus_id)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM)
            self._sample(True)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as e:  # NVML missing: report no samples rather than fail the bench
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _sample(self, with_reasons: bool):
        nv = self._nvml
        mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h) if with_reasons else None
        self.samples.append((mhz, reasons))

    def _run(self):
        if self.at_s is not None:
            t0 = time.perf_counter()
            for t in self.at_s:
                if self._stop.wait(max(0.0, t - (time.perf_counter() - t0))):
                    return
                try:
                    self._sample(True)
                except Exception:
                    return
            return
        k = 0
        while not self._stop.wait(self.period):
            k += 1
            try:
                self._sample(k % self.reasons_every == 0)
            except Exception:
                break

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        try:
            if self._nvml is not None:
                self._sample(True)
                self._nvml.nvmlShutdown()
        except Exception:
            pass

    def summary(self):
        bits = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}
        reasons = sorted({name for _, r in self.samples if r is not None for name, b in bits.items() if r & b})
        out = {"sm_mhz": statistics.median([m for m, _ in self.samples]) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
               "reason_samples": sum(1 for _, r in self.samples if r is not None), "source": "nvml",
               "gpu": "rank 0's"}
        if self.at_s is None:
            out["period_ms"] = self.period * 1e3
        else:
            out["schedule"] = ("one sample at entry and at exit, and during the timed region at "
                               + ", ".join(f"{t * 1e3:.1f} ms" for t in self.at_s)
                               + " (sparse: at N > 1 each NVML query stretches the step)")
        if self.error:
            out["error"] = self.error
        return out


def smi_id(dev) -> str:
    """PCI bus id of a torch device (NVML handle key), robust to CUDA_VISIBLE_DEVICES."""
    import torch
    p = torch.cuda.get_device_properties(dev)
    return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"


# ---------------------------------------------------------------- distributed plumbing

_T0 = time.perf_counter()


def progress(d, msg: str) -> None:
    """Phase timestamps on stderr (rank 0), so a slow or stuck multi-GPU run shows where it is."""
    if d.rank == 0:
        sys.stderr.write(f"[bench +{time.perf_counter() - _T0:.1f}s] {msg}\n")
        sys.stderr.flush()


class Dist:
    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if gpus != self.world:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}; launch N>1 with torch.distributed.run")

    def init(self):
        import torch
        torch.cuda.set_device(self.local)
        if self.world > 1:
            # NCCL prints a version banner on stdout unless told otherwise; rank 0's
            # only stdout line must be the JSON result.
            os.environ.setdefault("NCCL_DEBUG", "WARN")
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist.group.WORLD

    def barrier(self):
        if self.pg is not None:
            import torch.distributed as dist
            dist.barrier()

    def max(self, x: float) -> float:
        if self.pg is None:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            import torch.distributed as dist
            dist.destroy_process_group()


# ---------------------------------------------------------------- our arm

_INPUTS = {}


def make_inputs(rank: int):
    """Seeded host inputs for one shard (rank r owns rows [8192 r, 8192 (r+1))),
    generated once per process."""
    if rank in _INPUTS:
        return _INPUTS[rank]
    _INPUTS[rank] = _make_inputs(rank)
    return _INPUTS[rank]


def _make_inputs(rank: int):
    rng = np.random.default_rng(1_000 + rank)
    x = rng.standard_normal((ROWS, COLS), dtype=np.float32)
    y = rng.standard_normal((ROWS, COLS), dtype=np.float32)
    xi = rng.integers(-1000, 1001, (ROWS, COLS), dtype=np.int32)
    return x, y, xi


def run_ours(args, d: Dist):
    import torch
    from bee_b200 import _capi
    from bee_b200._capi import call

    d.init()
    progress(d, f"process group up ({d.world} ranks)")
    lib = _capi.lib()  # fails loudly if the CUDA library is missing
    dev = torch.device("cuda", d.local)
    stream = torch.cuda.Stream(device=dev)
    st = stream.cuda_stream
    peaks = load_peaks()

    x, y, xi = make_inputs(d.rank)
    progress(d, "inputs generated")
    hx = torch.from_numpy(x).pin_memory()
    hy = torch.from_numpy(y).pin_memory()
    hxi = torch.from_numpy(xi).pin_memory()
    with torch.cuda.stream(stream):
        dx = hx.to(dev, non_blocking=True)
        dy = hy.to(dev, non_blocking=True)
        dxi = hxi.to(dev, non_blocking=True)
        o_add = torch.empty_like(dx)
        o_mul = torch.empty_like(dx)
        o_bf = torch.empty((ROWS, COLS), dtype=torch.bfloat16, device=dev)
        o_rsum = torch.empty(ROWS, dtype=torch.float32, device=dev)
        o_rmax = torch.empty(ROWS, dtype=torch.float32, device=dev)
        o_sm = torch.empty_like(dx)
    stream.synchronize()

    F32, BF16, I32 = _capi.F32, _capi.BF16, _capi.I32
    # Across GPUs the int32 partials are combined by an NCCL all-reduce after the kernel
    # (default), or with --exchange peer inside the reduce kernel itself: its last block
    # stores the partial into every rank's CUDA IPC slot over NVLink and folds the world
    # partials in rank order (PeerReduce).  The peer exchange measures 0.576 ms per step at
    # N=2 against 0.595 with NCCL, but its spin-wait slows sharply while NVML is queried
    # on the GPU (the clock sampling the timed region needs), so NCCL is the default.
    peer = None
    if d.pg is not None and args.exchange == "peer":
        from bee_b200.shard import PeerReduce
        peer = PeerReduce(dev, group=d.pg)

    # step k writes its int32 sum into its own slot, so that the NCCL all-reduce of step k
    # (on a second stream, overlapping step k + 1) never races the next step's kernel
    ring = torch.zeros(args.warmup + args.steps + 1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    slot = [0]

    def sum_i32():
        dst = ring[slot[0]].data_ptr()
        if peer is not None:
            peer(0, I32, dxi.data_ptr(), N_EL, dst, st)
        else:
            call("bee_b200_reduce_global", 0, I32, dxi.data_ptr(), dst, N_EL, st)
    ops = [
        ("add_f32", lambda: call("bee_b200_ew_binary", 0, F32, dx.data_ptr(), dy.data_ptr(), o_add.data_ptr(), N_EL, st)),
        ("mul_f32", lambda: call("bee_b200_ew_binary", 2, F32, dx.data_ptr(), dy.data_ptr(), o_mul.data_ptr(), N_EL, st)),
        ("cast_f32_bf16", lambda: call("bee_b200_ew_cast", F32, dx.data_ptr(), BF16, o_bf.data_ptr(), N_EL, st)),
        ("row_sum_f32", lambda: call("bee_b200_reduce_axis", 0, F32, dx.data_ptr(), o_rsum.data_ptr(), ROWS, COLS, 1, st)),
        ("row_max_f32", lambda: call("bee_b200_reduce_axis", 2, F32, dx.data_ptr(), o_rmax.data_ptr(), ROWS, COLS, 1, st)),
        ("softmax_f32", lambda: call("bee_b200_softmax_rows", F32, dx.data_ptr(), o_sm.data_ptr(), ROWS, COLS, st)),
        ("sum_i32", sum_i32),
    ]
    launches_per_step = len(ops)

    comm = torch.cuda.Stream(device=dev) if (d.pg is not None and peer is None) else None

    def allreduce_isum(overlap=True):
        """Combines this step's int32 partials across GPUs: an NCCL all-reduce on the
        communication stream, after this step's kernels, overlapping the next step."""
        if comm is None:
            return
        import torch.distributed as dist
        if overlap:
            comm.wait_stream(stream)
            with torch.cuda.stream(comm):
                dist.all_reduce(ring[slot[0]], op=dist.ReduceOp.SUM)
        else:
            with torch.cuda.stream(stream):
                dist.all_reduce(ring[slot[0]], op=dist.ReduceOp.SUM)

    def step(k, evs=None):
        slot[0] = k
        for i, (_, fn) in enumerate(ops):
            if evs is not None:
                evs[i].record(stream)
            fn()
        if evs is not None:
            evs[len(ops)].record(stream)
        allreduce_isum()

    progress(d, "inputs resident, warm-up")
    # warm-up (also checks the int32 sum against the host, bit-exact); the last warm-up
    # step's duration places the clock samples inside the timed region at N > 1
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for k in range(args.warmup):
        if k == args.warmup - 1:
            w0.record(stream)
        step(k)
        if k == args.warmup - 1:
            w1.record(stream)
    if comm is not None:
        stream.wait_stream(comm)
    stream.synchronize()
    est_region_s = w0.elapsed_time(w1) / 1e3 * args.steps
    want = int(xi.astype(np.int64).sum())
    if d.pg is not None:
        import torch.distributed as dist
        t = torch.tensor([want], dtype=torch.int64, device=dev)
        dist.all_reduce(t)
        want = int(t.item())
    want32 = ((want + 2**31) % 2**32) - 2**31
    got = int(ring[args.warmup - 1].item())
    if got != want32:
        raise SystemExit(f"int32 sum mismatch: {got} != {want32}")

    # timed region
    per_step_events = [[torch.cuda.Event(enable_timing=True) for _ in range(len(ops) + 1)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d.barrier()
    torch.cuda.synchronize()
    # One sampler (its own process), on rank 0, for rank 0's GPU.
    # SM clock during the region.  N = 1: NVML every 2 ms (no measurable cost) and three
    # in-kernel probes.  N > 1: NVML in the process stretches the multi-GPU step even with
    # no query inside the region (N = 2: 0.570 ms per step without NVML, 0.882 ms with
    # NVML initialised and read just before and after the region, 0.572 ms with the
    # probes alone), so the clock during the region comes from the probes only
    # (bee_b200_clock_probe on a side stream: clock64 against the global timer for
    # 0.2 ms, a quarter, half and three quarters of the way through, on every rank) and
    # NVML is read once after the region for the throttle reasons.
    at_s = None
    probe_at = {args.steps // 4, args.steps // 2, (3 * args.steps) // 4}
    probe_buf = torch.zeros(len(probe_at), dtype=torch.float32, device=dev)
    probe_stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with ClockSampler(smi_id(dev), period_s=args.clock_period_ms / 1e3, reasons_every=args.clock_reasons_every,
                      enabled=not args.no_clocks and d.rank == 0 and args.clock_source != "probe"
                      and d.world == 1, at_s=at_s) as clk:
        t0.record(stream)
        np_i = 0
        for k in range(args.steps):
            if k in probe_at and not args.no_clocks and args.clock_source != "nvml":
                call("bee_b200_clock_probe", 200_000, probe_buf[np_i].data_ptr(), probe_stream.cuda_stream)
                np_i += 1
            # nothing between the kernels of a step: an event recorded between two
            # kernels would stop the next one's early (programmatic) launch
            step(args.warmup + k)
        if comm is not None:
            stream.wait_stream(comm)  # every step's exchange is inside the timed region
        t1.record(stream)
        stream.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    ms_local = t0.elapsed_time(t1)
    ms = d.max(ms_local)
    # Per-op breakdown (and the roofline's kernel duration): the same steps again,
    # with an event between ops; the events keep each kernel from starting before
    # the previous one ends, so this pass is slightly slower than the region above.
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(stream)
    for k in range(args.steps):
        step(args.warmup + k, per_step_events[k])
    if comm is not None:
        stream.wait_stream(comm)
    b1.record(stream)
    stream.synchronize()
    d.barrier()
    breakdown_ms_per_step = d.max(b0.elapsed_time(b1)) / args.steps
    per_op_ms = {name: sum(ev[i].elapsed_time(ev[i + 1]) for ev in per_step_events) / args.steps
                 for i, (name, _) in enumerate(ops)}
    if d.world > 1:
        import torch.distributed as dist
        t = torch.tensor([per_op_ms[n] for n, _ in ops], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        per_op_ms = {n: float(v) for (n, _), v in zip(ops, t.tolist())}

    # Each op alone (outside the timed region): the same kernel 3 + 10 times back to back,
    # so no other op's dirty L2 lines are written back during it.  Inside the step, a
    # reader that follows a writer (row sum after the cast, the int32 sum after the
    # softmax) also moves the writer's last ~30-40 MB of dirty lines to DRAM.
    alone_ms = {}
    slot[0] = ring.numel() - 1
    for name, fn in ops:
        if name == "sum_i32":  # the local reduce alone, without the cross-GPU exchange
            fn = lambda: call("bee_b200_reduce_global", 0, I32, dxi.data_ptr(), ring[slot[0]].data_ptr(), N_EL, st)
        for _ in range(3):
            fn()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(10):
            fn()
        a1.record(stream)
        stream.synchronize()
        alone_ms[name] = a0.elapsed_time(a1) / 10
    if d.world > 1:
        import torch.distributed as dist
        t = torch.tensor([alone_ms[n] for n, _ in ops], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        alone_ms = {n: float(v) for (n, _), v in zip(ops, t.tolist())}

    ms_per_step = ms / args.steps
    value = d.world * STEP_BYTES * args.steps / (ms / 1e3) / 1e9
    dominant = max(per_op_ms, key=per_op_ms.get)
    dom_gbs = OP_BYTES[dominant] / (per_op_ms[dominant] / 1e3) / 1e9

    # end to end through the C ABI with host buffers: H2D inputs, ops, D2H outputs
    e2e = None
    if not args.no_e2e:
        slot[0] = ring.numel() - 1  # a slot of its own, exchanged on the compute stream
        progress(d, "sweep timed; e2e")
        e2e = run_e2e(args, d, dev, stream, hx, hy, hxi, [dx, dy, dxi],
                      [o_add, o_mul, o_bf, o_rsum, o_rmax, o_sm, ring[slot[0]:slot[0] + 1]])

    clocks = clk.summary()
    probe_stream.synchronize()
    probe_mhz = [round(v, 1) for v in probe_buf[:np_i].tolist()] if not args.no_clocks else []
    if d.world > 1 and probe_mhz:
        import torch.distributed as dist
        t = torch.tensor(probe_mhz, dtype=torch.float64, device=dev)
        lo = t.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)  # the slowest clock any rank saw at each probe
        probe_mhz = [round(v, 1) for v in lo.tolist()]
    if probe_mhz:
        clocks["probe_mhz_during"] = probe_mhz
    if d.world > 1 and not args.no_clocks:
        clocks = {"sm_mhz": statistics.median(probe_mhz) if probe_mhz else None, "probe_mhz_during": probe_mhz,
                  "sm_mhz_source": "median of in-kernel probes during the timed region (min over ranks)"}
        # the NVML read for the throttle reasons waits until every measurement of this run
        # (extras included) is done: NVML in the process slows multi-GPU steps
    if peer is not None:
        peer.close()
    progress(d, "extras")
    extra = None if args.no_extras else run_extras(args, d, dev, stream, peaks)
    progress(d, "extras done")
    if d.world > 1 and not args.no_clocks and d.rank == 0:
        after = ClockSampler(smi_id(dev), enabled=True)
        with after:
            pass  # one NVML read (clock, throttle reasons), after every measurement of the run
        s_after = after.summary()
        clocks.update({"sm_max_mhz": s_after.get("sm_max_mhz"), "reasons": s_after.get("reasons", []),
                       "nvml_after_run": {"sm_mhz": s_after.get("sm_mhz"), "reasons": s_after.get("reasons"),
                                          "error": s_after.get("error")},
                       "reasons_source": "NVML read on rank 0's GPU after the run's measurements"})
    out = None
    if d.rank == 0:
        ops_json = {n: {"ms": round(per_op_ms[n], 4), "GB/s": round(OP_BYTES[n] / (per_op_ms[n] / 1e3) / 1e9, 1),
                        "frac_of_hbm": round(OP_BYTES[n] / (per_op_ms[n] / 1e3) / 1e9 / peaks["hbm_gbs"], 3),
                        "alone_ms": round(alone_ms[n], 4),
                        "alone_frac_of_hbm": round(OP_BYTES[n] / (alone_ms[n] / 1e3) / 1e9 / peaks["hbm_gbs"], 3)}
                    for n, _ in ops}
        ops_note = ("ms / frac_of_hbm: a second pass of the same steps with an event between ops "
                    f"({round(breakdown_ms_per_step, 4)} ms per step; the events also stop each kernel's early "
                    "launch), where a reader that follows a writer also writes the writer's dirty L2 lines back "
                    "to DRAM; alone_*: the same kernel repeated back to back after the timed region")
        out = {
            "metric": "memory-bound op sweep HBM GB/s (add, mul, fp32->bf16 cast, row sum, row max, row softmax, "
                      "int32 full sum) on [8192, 8192] row shards",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": d.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded N(0,1) fp32, uniform int32 in [-1000, 1000])",
            "config": sweep_config(d.world, peer is not None),
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": round(dom_gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(dom_gbs / peaks["hbm_gbs"], 3),
                         "peak_source": peaks["source"], "algorithmic_bytes": OP_BYTES[dominant],
                         "traffic": NCU_TRAFFIC.get(dominant),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch"},
            "ops": ops_json,
            "ops_note": ops_note,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "e2e": e2e,
            "extra": extra,
        }
    return out


def run_extras(args, d, dev, stream, peaks):
    """The other configs of the path, each timed on its own (CUDA events on the
    launching stream, max over ranks) after the headline sweep, the memory-bound ones
    first: after the 8192^3 GEMMs, which run at the 1000 W power cap, the SM clock
    stays low for longer than a warm-up (each config reports the SM clock an
    in-kernel probe saw during its timed region, ``sm_mhz_probe``):

    * gemm_bf16_8192: C = A.B, M = N = K = 8192, bf16 in, fp32 accumulate, bf16 out;
      B sharded by output columns (each GPU owns an [8192, 8192] column block of a
      [8192, 8192*N] B, weak scaling, no collective);
    * gemm_bf16_8192_splitk: the same single 8192^3 product with K sharded over the
      GPUs (strong scaling): the GEMM epilogue stores fp32 partial tiles into the
      owning GPU over NVLink, the owner sums, casts and writes its tiles into every
      GPU's C (SplitKGemm); the unfused chain (fp32 partial, NCCL all-reduce,
      cast) is timed beside it;
    * rms_norm_rope_bf16: RMSNorm (eps 1e-6) + RoPE (theta 1e4, rotate-half) of X
      [16 x 2048, 4096] bf16 viewed [16, 2048, 32, 128], fused, per GPU (weak);
    * attention_bf16: S = Q.K^T/sqrt(128) (fp32), P = softmax(S) (bf16),
      O = P.V for 32 heads x [2048, 128] per GPU (heads sharded, weak);
    * gemm_f16_8192: the gemm_bf16_8192 product with f16 inputs and output;
    * gemm_f32_1024: the fp32 parity config, 1024^3.
    """
    import torch
    from bee_b200 import _capi
    from bee_b200._capi import call
    from bee_b200.shard import shard_range
    st = stream.cuda_stream
    steps = max(3, min(args.steps, 20))
    warm = 3
    only = getattr(args, "only", None)

    def want(*names):
        return only is None or only in names
    g = torch.Generator(device=dev).manual_seed(4321 + d.rank)
    out = {}

    probe_buf = torch.zeros(1, dtype=torch.float32, device=dev)
    probe_stream = torch.cuda.Stream(device=dev)
    probe_log = {}

    def timed(fn, label=None):
        """ms per call of fn.  Warm-up: at least `warm` calls and about 30 ms of work, so
        that the SM clock has recovered from the previous config (the 8192^3 GEMMs run at
        the 1000 W power cap); the timed region: at least `steps` calls and about 10 ms by
        a warm estimate (so the 0.2 ms clock probe stays small beside it).
        Call counts come from the slowest rank's estimate, so every rank makes the same
        calls (fn may hold collectives).  With a label, one in-kernel clock probe
        (0.2 ms on a side stream) runs mid-region and its SM MHz is reported."""
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        fn()
        e1.record(stream)
        stream.synchronize()
        est = max(d.max(e0.elapsed_time(e1)), 1e-3)  # the first call may carry one-time costs
        n_warm = max(warm, min(int(30.0 / est), 2000))
        for _ in range(n_warm):
            fn()
        e0.record(stream)
        for _ in range(3):
            fn()
        e1.record(stream)
        stream.synchronize()
        est = max(d.max(e0.elapsed_time(e1)) / 3, 1e-3)  # warm estimate sizes the region
        n_time = max(steps, min(int(10.0 / est), 2000))
        d.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(n_time):
            if label is not None and i == n_time // 2 and not args.no_clocks:
                call("bee_b200_clock_probe", 200_000, probe_buf.data_ptr(), probe_stream.cuda_stream)
            fn()
        e1.record(stream)
        stream.synchronize()
        if label is not None and not args.no_clocks:
            probe_stream.synchronize()
            probe_log[label] = round(float(probe_buf.item()), 1)
        ms_call = d.max(e0.elapsed_time(e1)) / n_time
        progress(d, f"extra {label or 'config'}: {ms_call:.4f} ms per call ({n_warm} warm-up, {n_time} timed)")
        return ms_call

    def status_ok():
        import ctypes
        c = ctypes.c_int(-1)
        call("bee_b200_device_status", ctypes.byref(c))
        return c.value == 0

    with torch.cuda.stream(stream):
        if want("rms_norm_rope_bf16"):
            rows, cols, seq, heads, hd = 16 * 2048, 4096, 2048, 32, 128
            x = torch.randn(rows, cols, device=dev, generator=g).to(torch.bfloat16)
            w = (1 + 0.02 * torch.randn(cols, device=dev, generator=g)).to(torch.bfloat16)
            y = torch.empty_like(x)
            ms = timed(lambda: call("bee_b200_rms_norm_rope", _capi.BF16, x.data_ptr(), w.data_ptr(), y.data_ptr(), rows,
                                    seq, heads, hd, 1e-6, 10000.0, 0, st), label="rms_norm_rope_bf16")
            nbytes = 2 * rows * cols * 2 + cols * 2
            gbs = d.world * nbytes / (ms / 1e3) / 1e9
            out["rms_norm_rope_bf16"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "unit": "GB/s",
                                         "frac_of_hbm": round(gbs / d.world / peaks["hbm_gbs"], 3),
                                         "bytes_per_gpu": nbytes, "scaling": "weak (rows sharded)"}
            del x, w, y
        if want("gemm_f32_1024"):
            a32 = torch.rand(1024, 1024, device=dev, generator=g) * 2 - 1
            b32 = torch.rand(1024, 1024, device=dev, generator=g) * 2 - 1
            c32 = torch.empty_like(a32)
            ms = timed(lambda: call("bee_b200_matmul", _capi.F32, a32.data_ptr(), b32.data_ptr(), c32.data_ptr(), 1024,
                                    1024, 1024, st), label="gemm_f32_1024")
            out["gemm_f32_1024"] = {"ms": round(ms, 4), "TFLOP/s": round(2.0 * 1024 ** 3 / (ms / 1e3) / 1e12, 2),
                                    "unit": "TFLOP/s (per GPU)",
                                    "path": "fp32 as three bf16 pieces, six products on the tcgen05 tensor cores, "
                                            "fp32 accumulate (parity config, rel tol 1e-4)"}
            del a32, b32, c32
        if want("transpose_f32_8192", "bcast_sub_rowmax_f32_8192", "sum_dim0_f32_8192", "contiguous_kt_bf16"):
            # layout and broadcast ops on the [8192, 8192] fp32 shard (HBM-bound, 2 x 256 MiB moved)
            import ctypes
            x = torch.randn(8192, 8192, device=dev, generator=g)
            y = torch.empty_like(x)
            ms = timed(lambda: call("bee_b200_transpose_2d", _capi.F32, x.data_ptr(), y.data_ptr(), 8192, 8192, st),
                       label="transpose_f32_8192")
            nbytes = 2 * 8192 * 8192 * 4
            gbs = d.world * nbytes / (ms / 1e3) / 1e9
            out["transpose_f32_8192"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "unit": "GB/s",
                                         "frac_of_hbm": round(gbs / d.world / peaks["hbm_gbs"], 3),
                                         "bytes_per_gpu": nbytes, "scaling": "weak"}
            rmax = torch.empty(8192, device=dev)
            call("bee_b200_reduce_axis", _capi.MAX, _capi.F32, x.data_ptr(), rmax.data_ptr(), 8192, 8192, 1, st)
            shp = (ctypes.c_int64 * 2)(8192, 8192)
            sa = (ctypes.c_int64 * 2)(8192, 1)
            sb = (ctypes.c_int64 * 2)(1, 0)
            ms = timed(lambda: call("bee_b200_ew_binary_strided", _capi.SUB, _capi.F32, 2, shp, x.data_ptr(), sa,
                                    rmax.data_ptr(), sb, y.data_ptr(), st), label="bcast_sub_rowmax_f32_8192")
            nbytes = 2 * 8192 * 8192 * 4 + 8192 * 4
            gbs = d.world * nbytes / (ms / 1e3) / 1e9
            out["bcast_sub_rowmax_f32_8192"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "unit": "GB/s",
                                                "frac_of_hbm": round(gbs / d.world / peaks["hbm_gbs"], 3),
                                                "op": "x[8192, 8192] - rowmax[8192, 1] (broadcast, stride 0)",
                                                "bytes_per_gpu": nbytes, "scaling": "weak"}
            colsum = torch.empty(8192, device=dev)
            ms = timed(lambda: call("bee_b200_reduce_axis", _capi.SUM, _capi.F32, x.data_ptr(), colsum.data_ptr(), 1, 8192,
                                    8192, st), label="sum_dim0_f32_8192")
            nbytes = 8192 * 8192 * 4 + 8192 * 4
            gbs = d.world * nbytes / (ms / 1e3) / 1e9
            out["sum_dim0_f32_8192"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "unit": "GB/s",
                                        "frac_of_hbm": round(gbs / d.world / peaks["hbm_gbs"], 3),
                                        "op": "sum(x, 0) of [8192, 8192] fp32 (column reduce, axis split over CTAs)",
                                        "bytes_per_gpu": nbytes, "scaling": "weak"}
            del colsum
            kq = torch.randn(256, 2048, 128, device=dev, generator=g).to(torch.bfloat16)
            kt = torch.empty(256, 128, 2048, device=dev, dtype=torch.bfloat16)
            vsh = (ctypes.c_int64 * 3)(256, 128, 2048)
            vst = (ctypes.c_int64 * 3)(2048 * 128, 1, 128)
            ms = timed(lambda: call("bee_b200_strided_copy", _capi.BF16, kq.data_ptr(), 3, vsh, vst, kt.data_ptr(), st),
                       label="contiguous_kt_bf16")
            nbytes = 2 * 256 * 2048 * 128 * 2
            gbs = d.world * nbytes / (ms / 1e3) / 1e9
            out["contiguous_kt_bf16"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "unit": "GB/s",
                                         "frac_of_hbm": round(gbs / d.world / peaks["hbm_gbs"], 3),
                                         "op": "contiguous() of K^T, K [256, 2048, 128] bf16 (128 MiB each way)",
                                         "bytes_per_gpu": nbytes, "scaling": "weak"}
            del x, y, rmax, kq, kt

        if want("attention_bf16"):
            h, s_, dh = 32, 2048, 128
            q = torch.randn(h, s_, dh, device=dev, generator=g).to(torch.bfloat16)
            k = torch.randn(h, s_, dh, device=dev, generator=g).to(torch.bfloat16)
            v = torch.randn(h, s_, dh, device=dev, generator=g).to(torch.bfloat16)
            S = torch.empty(h, s_, s_, device=dev, dtype=torch.float32)
            P = torch.empty(h, s_, s_, device=dev, dtype=torch.bfloat16)
            o = torch.empty(h, s_, dh, device=dev, dtype=torch.bfloat16)
            scale = 1.0 / np.sqrt(dh)

            def attention_chain():
                call("bee_b200_bmm", _capi.BF16, _capi.F32, q.data_ptr(), k.data_ptr(), S.data_ptr(), h, s_, dh, s_, 1,
                     scale, st)
                call("bee_b200_softmax_rows_to", _capi.F32, S.data_ptr(), _capi.BF16, P.data_ptr(), h * s_, s_, st)
                call("bee_b200_bmm", _capi.BF16, _capi.BF16, P.data_ptr(), v.data_ptr(), o.data_ptr(), h, s_, s_, dh, 0,
                     1.0, st)

            def attention_fused():
                call("bee_b200_attention", _capi.BF16, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), h, s_, dh,
                     scale, st)
            aflop = 2.0 * 2 * h * s_ * s_ * dh
            ms = timed(attention_fused, label="attention_bf16")
            tf = d.world * aflop / (ms / 1e3) / 1e12
            ms_c = timed(attention_chain)
            tf_c = d.world * aflop / (ms_c / 1e3) / 1e12
            out["attention_bf16"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1), "unit": "TFLOP/s",
                                     "frac_of_measured_bf16_burst": round(tf / d.world / peaks["bf16_tflops"], 3),
                                     "kernels": "fused (scores and probabilities stay on chip)",
                                     "unfused_chain": {"ms": round(ms_c, 4), "TFLOP/s": round(tf_c, 1),
                                                       "kernels": "bmm (QK^T, fp32 out) -> softmax fp32->bf16 -> bmm (PV)"},
                                     "scaling": "weak (heads sharded)", "status_ok": status_ok()}
            del q, k, v, S, P, o
        if want("gemm_bf16_8192", "gemm_bf16_8192_splitk", "gemm_f16_8192"):
            n = 8192
            std = (1.0 / np.sqrt(n)) ** 0.5  # N(0, variance 1/sqrt(8192))
            a = (torch.randn(n, n, device=dev, generator=g) * std).to(torch.bfloat16)
            b = (torch.randn(n, n, device=dev, generator=g) * std).to(torch.bfloat16)
            c = torch.empty(n, n, device=dev, dtype=torch.bfloat16)
            flop = 2.0 * n ** 3
            ms = timed(lambda: call("bee_b200_bmm", _capi.BF16, _capi.BF16, a.data_ptr(), b.data_ptr(), c.data_ptr(),
                                    1, n, n, n, 0, 1.0, st), label="gemm_bf16_8192")
            tf = d.world * flop / (ms / 1e3) / 1e12
            out["gemm_bf16_8192"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1), "unit": "TFLOP/s",
                                     "frac_of_measured_bf16_burst": round(tf / d.world / peaks["bf16_tflops"], 3),
                                     "frac_of_measured_bf16_sustained": round(tf / d.world / peaks["bf16_tflops_sustained"], 3),
                                     "frac_of_spec_2250": round(tf / d.world / 2250.0, 3),
                                     "scaling": "weak (column shards)", "status_ok": status_ok()}
            if want("gemm_f16_8192"):
                # the same product with f16 A and B (f16 out): the tensor cores' f16 operand format
                a16, b16 = a.to(torch.float16), b.to(torch.float16)
                c16 = torch.empty(n, n, device=dev, dtype=torch.float16)
                ms16 = timed(lambda: call("bee_b200_bmm", _capi.F16, _capi.F16, a16.data_ptr(), b16.data_ptr(),
                                          c16.data_ptr(), 1, n, n, n, 0, 1.0, st), label="gemm_f16_8192")
                tf16 = d.world * flop / (ms16 / 1e3) / 1e12
                out["gemm_f16_8192"] = {"ms": round(ms16, 4), "TFLOP/s": round(tf16, 1), "unit": "TFLOP/s",
                                        "frac_of_measured_bf16_burst": round(tf16 / d.world / peaks["bf16_tflops"], 3),
                                        "scaling": "weak (column shards)", "status_ok": status_ok()}
                del a16, b16, c16

            # split-K: rank r multiplies A[:, K_r] by B[K_r, :]
            klo, khi = shard_range(n, d.world, d.rank)
            kr = khi - klo
            ak = a[:, klo:khi].contiguous()
            bk = b[klo:khi].contiguous()
            part = torch.empty(n, n, device=dev, dtype=torch.float32)

            def splitk():
                call("bee_b200_bmm", _capi.BF16, _capi.F32, ak.data_ptr(), bk.data_ptr(), part.data_ptr(), 1, n, kr, n,
                     0, 1.0, st)
                if d.pg is not None:
                    import torch.distributed as dist
                    dist.all_reduce(part, op=dist.ReduceOp.SUM)
                call("bee_b200_ew_cast", _capi.F32, part.data_ptr(), _capi.BF16, c.data_ptr(), n * n, st)
            ms_nccl = timed(splitk)
            del ak, bk, part

            from bee_b200.shard import SplitKGemm
            fused = SplitKGemm(n, n, dev, group=d.pg)
            a_ptr = a.data_ptr() + 2 * klo
            b_ptr = b[klo:khi].data_ptr()
            ms = timed(lambda: fused(a_ptr, n, b_ptr, kr, st), label="gemm_bf16_8192_splitk")
            ok_fused = status_ok()
            fused.close()
            tf = flop / (ms / 1e3) / 1e12
            tf_nccl = flop / (ms_nccl / 1e3) / 1e12
            owned = -(-(n // 256) ** 2 // d.world)
            out["gemm_bf16_8192_splitk"] = {
                "ms": round(ms, 4), "TFLOP/s": round(tf, 1), "unit": "TFLOP/s",
                "scaling": "strong (K sharded)",
                "kernels": "tcgen05 GEMM whose epilogue stores fp32 partial tiles into the owner GPU over NVLink, "
                           "owner reduce writing bf16 C into every GPU; two one-element NCCL all-reduces as barriers",
                "nvlink_bytes_out_per_gpu": (d.world - 1) * owned * 256 * 256 * (4 + 2) if d.world > 1 else 0,
                "status_ok": ok_fused,
                "nccl_allreduce_chain": {"ms": round(ms_nccl, 4), "TFLOP/s": round(tf_nccl, 1),
                                         "kernels": "bmm fp32 out -> NCCL all-reduce (fp32) -> cast",
                                         "allreduce_bytes_per_gpu": n * n * 4 if d.world > 1 else 0}}
            del a, b, c
        if want("bridge_matmul") and d.world == 1:
            # plumbing cost around a matmul through the C++ bridge (bee_b200/host/bridge_bench.cpp),
            # on the same GPU (the child inherits the device selection)
            exe = ROOT / "bee_b200" / "_lib" / "bridge_bench"
            if exe.exists():
                stream.synchronize()
                r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
                if r.returncode == 0:
                    res = json.loads(r.stdout.strip().splitlines()[-1])
                    res["what"] = ("allocate C + zero fill + matmul + free, every call synchronous (the reference's "
                                   "bridge sequence) vs the asynchronous bridge (pool allocation, no fill) with one "
                                   "fence per call, and pipelined")
                    out["bridge_matmul"] = res
                else:
                    out["bridge_matmul"] = {"error": (r.stderr or r.stdout)[-300:]}
    stream.synchronize()
    for label, mhz in probe_log.items():
        if isinstance(out.get(label), dict):
            out[label]["sm_mhz_probe"] = mhz
    return out


def run_e2e(args, d, dev, stream, hx, hy, hxi, dins, outs):
    """Same sweep through the C ABI with host buffers: every step copies the
    inputs host->device (pinned), runs the ops and copies every output back.

    Two device buffer sets (inputs and outputs) alternate between steps, as a
    caller streaming batches would arrange it, and the copies go on two copy
    streams, so PCIe carries both directions for the whole step: the upload of
    step k+1's inputs and the download of step k's outputs run together, and
    step k+1's kernels need only their own upload (the download reading the
    other buffer set).  A buffer set is reused only after its download and its
    kernels are done.  The timed region ends when the last step's outputs are
    in host memory."""
    import torch
    from bee_b200 import _capi
    from bee_b200._capi import call
    st = stream.cuda_stream
    F32, BF16, I32 = _capi.F32, _capi.BF16, _capi.I32
    sets = [(list(dins), list(outs)), ([torch.empty_like(t) for t in dins], [torch.empty_like(t) for t in outs])]
    h_outs = [[torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs] for _ in range(2)]
    h_ins = [hx, hy, hxi]
    h2d = sum(t.numel() * t.element_size() for t in h_ins)
    d2h = sum(t.numel() * t.element_size() for t in h_outs[0])

    def run_ops(k):
        (dx, dy, dxi), (o_add, o_mul, o_bf, o_rsum, o_rmax, o_sm, o_isum) = sets[k]
        call("bee_b200_ew_binary", 0, F32, dx.data_ptr(), dy.data_ptr(), o_add.data_ptr(), N_EL, st)
        call("bee_b200_ew_binary", 2, F32, dx.data_ptr(), dy.data_ptr(), o_mul.data_ptr(), N_EL, st)
        call("bee_b200_ew_cast", F32, dx.data_ptr(), BF16, o_bf.data_ptr(), N_EL, st)
        call("bee_b200_reduce_axis", 0, F32, dx.data_ptr(), o_rsum.data_ptr(), ROWS, COLS, 1, st)
        call("bee_b200_reduce_axis", 2, F32, dx.data_ptr(), o_rmax.data_ptr(), ROWS, COLS, 1, st)
        call("bee_b200_softmax_rows", F32, dx.data_ptr(), o_sm.data_ptr(), ROWS, COLS, st)
        call("bee_b200_reduce_global", 0, I32, dxi.data_ptr(), o_isum.data_ptr(), N_EL, st)
        if d.pg is not None:
            import torch.distributed as dist
            with torch.cuda.stream(stream):
                dist.all_reduce(o_isum, op=dist.ReduceOp.SUM)

    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_up = [torch.cuda.Event() for _ in range(2)]
    ev_ops = [torch.cuda.Event() for _ in range(2)]
    ev_down = [torch.cuda.Event() for _ in range(2)]
    for k in range(2):  # every set starts free
        ev_ops[k].record(stream)
        ev_down[k].record(stream)

    def e2e_step(i):
        k = i & 1
        ins, outs_k = sets[k]
        up.wait_event(ev_ops[k])  # this set's previous kernels have read their inputs
        for h, dd in zip(h_ins, ins):
            call("bee_b200_memcpy_h2d", dd.data_ptr(), h.data_ptr(), h.numel() * h.element_size(), up.cuda_stream)
        ev_up[k].record(up)
        stream.wait_event(ev_up[k])
        stream.wait_event(ev_down[k])  # this set's previous outputs are in host memory
        run_ops(k)
        ev_ops[k].record(stream)
        down.wait_event(ev_ops[k])
        for h, o in zip(h_outs[k], outs_k):
            call("bee_b200_memcpy_d2h", h.data_ptr(), o.data_ptr(), o.numel() * o.element_size(), down.cuda_stream)
        ev_down[k].record(down)

    steps = max(2, min(args.steps, 6))
    for i in range(2):  # warm-up, both sets
        e2e_step(i)
    for k in range(2):
        stream.wait_event(ev_down[k])
    d.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    up.wait_event(t0)
    down.wait_event(t0)
    for i in range(steps):
        e2e_step(i)
    for k in range(2):
        stream.wait_event(ev_down[k])
    t1.record(stream)
    call("bee_b200_stream_synchronize", st)
    ms = d.max(t0.elapsed_time(t1))
    # each direction alone (same copies, one stream, nothing else running)
    def one_way(copy_fn, nbytes):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(up)
        for _ in range(2):
            copy_fn()
        b.record(up)
        b.synchronize()
        return round(2 * nbytes / (a.elapsed_time(b) / 1e3) / 1e9, 1)
    h2d_alone = one_way(lambda: [call("bee_b200_memcpy_h2d", dd.data_ptr(), h.data_ptr(), h.numel() * h.element_size(),
                                      up.cuda_stream) for h, dd in zip(h_ins, sets[0][0])], h2d)
    d2h_alone = one_way(lambda: [call("bee_b200_memcpy_d2h", h.data_ptr(), o.data_ptr(), o.numel() * o.element_size(),
                                      up.cuda_stream) for h, o in zip(h_outs[0], sets[0][1])], d2h)
    # the last step's results, read back, must match the device-timed sweep's
    ok = all(torch.equal(h.to(dev), o) for h, o in zip(h_outs[(steps - 1) & 1], sets[(steps - 1) & 1][1]))
    return {"value": round(d.world * STEP_BYTES * steps / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "ms_per_step": round(ms / steps, 3), "outputs_match_device": bool(ok),
            "pcie_gbs": {"h2d_alone": h2d_alone, "d2h_alone": d2h_alone,
                         "both_in_step": round((h2d + d2h) / (ms / steps / 1e3) / 1e9, 1)},
            "copies": "pinned host buffers, two device buffer sets alternating between steps; H2D of step k+1 and "
                      "D2H of step k on two copy streams at once"}


# ---------------------------------------------------------------- CPU baseline / reference arm

def cpu_sweep(sample_rows: int, reps: int = 1):
    """Times the reference CPU ops (oracle/_ref, else the oracle port) on a
    [sample_rows, 8192] sample of the shard; returns (GB/s, info)."""
    from oracle.oracle import Oracle, Reference, reference_available
    x, y, xi = make_inputs(0)
    xs, ys, xis = x[:sample_rows], y[:sample_rows], xi[:sample_rows]
    n = sample_rows * COLS
    scale = sample_rows / ROWS
    times = {}
    if reference_available():
        ref = Reference()
        kind, cores, isa = "reference", ref.threads(), ref.isa()
        xs, ys, xis = (np.ascontiguousarray(v) for v in (xs, ys, xis))
        _INPUTS[("ref", sample_rows)] = (xs, ys, xis)  # kept alive: the reference caches its Tensors by address
        times.update(ref.sweep(xs, ys, xis)[1])
        # the reference's CPU cast to BF16 writes nothing (CastCpu.hpp:348): time the restatement
        orc = Oracle()
        t = time.perf_counter()
        orc.cast_f32_bf16(xs)
        times["cast_f32_bf16"] = time.perf_counter() - t
    else:
        orc = Oracle()
        kind, cores, isa = "port", 1, "scalar C (oracle port)"

        def tm(fn):
            t = time.perf_counter()
            fn()
            return time.perf_counter() - t
        times["add_f32"] = tm(lambda: orc.binary(0, xs, ys))
        times["mul_f32"] = tm(lambda: orc.binary(2, xs, ys))
        times["cast_f32_bf16"] = tm(lambda: orc.cast_f32_bf16(xs))
        times["row_sum_f32"] = tm(lambda: orc.reduce_rows_f32(0, xs))
        times["row_max_f32"] = tm(lambda: orc.reduce_rows_f32(2, xs))
        times["softmax_f32"] = tm(lambda: orc.softmax_f32(xs))
        times["sum_i32"] = tm(lambda: orc.reduce_global_i32(0, xis))
    total_t = sum(times.values())
    gbs = STEP_BYTES * scale / total_t / 1e9
    info = {"kind": kind, "cores": cores, "isa": isa,
            "sample": f"[{sample_rows}, {COLS}] rows of the [8192, 8192] shard per op ({n} elements), "
                      f"all 7 ops; bf16 cast timed on the oracle restatement (the reference's CPU cast to BF16 "
                      f"is a no-op)" if kind == "reference" else f"[{sample_rows}, {COLS}] sample, oracle port",
            "per_op_s": {k: round(v, 4) for k, v in times.items()}}
    return gbs, info


def run_reference(args, d: Dist):
    if d.rank != 0:
        return None
    sample_rows = args.ref_rows
    for _ in range(args.warmup):
        cpu_sweep(sample_rows)
    vals, info = [], None
    t_all = time.perf_counter()
    for _ in range(args.steps):
        v, info = cpu_sweep(sample_rows)
        vals.append(v)
    wall = time.perf_counter() - t_all
    value = statistics.median(vals)
    cb = dict(info)
    cb.update({"value": round(value, 3), "unit": "GB/s"})
    return {
        "metric": "memory-bound op sweep HBM GB/s (add, mul, fp32->bf16 cast, row sum, row max, row softmax, "
                  "int32 full sum) on [8192, 8192] row shards",
        "impl": "reference", "value": round(value, 3), "unit": "GB/s", "n_gpus": d.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(wall / max(args.steps, 1) * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) fp32, uniform int32 in [-1000, 1000])",
        "config": sweep_config(d.world, args.exchange == "peer"),
        "cpu_baseline": cb,
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["sweep"], default="sweep")
    ap.add_argument("--ref-rows", type=int, default=ROWS,
                    help="rows of the [8192, 8192] shard per CPU step (default: the whole shard)")
    ap.add_argument("--cpu-reps", type=int, default=8, help="CPU-baseline steps timed in the GPU arm (rank 0, N=1)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the GEMM / RMSNorm+RoPE / attention configs")
    ap.add_argument("--no-clocks", action="store_true", help="do not sample SM clocks during the timed region")
    ap.add_argument("--clock-period-ms", type=float, default=2.0, help="SM clock sampling period")
    ap.add_argument("--clock-reasons-every", type=int, default=10,
                    help="query the throttle reasons every this many clock samples")
    ap.add_argument("--clock-source", choices=["both", "nvml", "probe"], default="both",
                    help="SM clock evidence: NVML samples, in-kernel probes, or both")
    ap.add_argument("--exchange", choices=["nccl", "peer"], default="nccl",
                    help="how the int32 partial sums are combined across GPUs")
    ap.add_argument("--only", default=None,
                    help="profiling mode: run only the named extra config (e.g. attention_bf16) and print its timing")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    d = Dist(args.gpus)
    if args.impl == "reference":
        out = run_reference(args, d)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    if args.only:
        import torch
        d.init()
        dev = torch.device("cuda", d.local)
        stream = torch.cuda.Stream(device=dev)
        extra = run_extras(args, d, dev, stream, load_peaks())
        if d.rank == 0:
            print(json.dumps({"only": args.only, "extra": extra}), flush=True)
        d.close()
        return
    try:
        out = run_ours(args, d)
        if out is not None and not args.no_cpu_baseline and d.world == 1:
            cpu_sweep(args.ref_rows)  # warm-up (thread pool, first touch)
            runs = [cpu_sweep(args.ref_rows) for _ in range(max(args.cpu_reps, 1))]
            gbs = statistics.median(g for g, _ in runs)
            cb = dict(runs[-1][1])
            cb.update({"value": round(gbs, 3), "unit": "GB/s", "steps": len(runs),
                       "statistic": "median over the steps"})
            out["cpu_baseline"] = cb
        if out is not None:
            print(json.dumps(out), flush=True)
    finally:
        d.close()


if __name__ == "__main__":
    main()
