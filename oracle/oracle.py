"""numpy-facing wrappers of the oracle libraries.

TEST INFRASTRUCTURE ONLY (the checker): tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg use it; the bee_b200 product never does.

* ``Oracle`` wraps ``oracle/_build/liboracle.so`` — our C restatement of the
  reference algorithms (oracle/bee_oracle.c), plus numpy restatements of the
  elementwise ops (IEEE fp32 arithmetic is the same on both sides).
* ``Reference`` wraps ``oracle/_ref/libbee_ref.so`` — the reference's own CPU
  path (Bee::Tensor public ops) compiled by oracle/Makefile; present wherever
  the library was built (it travels with the repository snapshot).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libbee_ref.so"

_vp, _i64, _i, _f, _d = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_double


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def build_oracle() -> Path:
    if not ORACLE_SO.exists() or ORACLE_SO.stat().st_mtime < (HERE / "bee_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return ORACLE_SO


# ------------------------------------------------------------------ bf16 helpers

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit pattern (NaN -> 0x7fff), as uint16."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (returned as fp32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ------------------------------------------------------------------ f16 helpers
# IEEE binary16 with round-to-nearest-even, the definition the f16 paths are
# pinned to (the reference stores F16 but computes nothing in it,
# Bee/Tensor/Core/DType.hpp:10-15).

def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


def matmul_exact(a: np.ndarray, b: np.ndarray, b_trans: bool = False, alpha: float = 1.0) -> np.ndarray:
    """alpha * A.op(B) in float64 for batched [batch, M, K] x [batch, K, N]
    operands (op(B) = B^T of [batch, N, K] when b_trans): the exact product of
    16-bit inputs to within float64 rounding, which an fp32-accumulating kernel
    must match within its tolerance."""
    a64 = np.asarray(a, np.float64)
    b64 = np.asarray(b, np.float64)
    if b_trans:
        b64 = np.swapaxes(b64, -1, -2)
    return alpha * (a64 @ b64)


class Oracle:
    """Our C restatement of the reference algorithms (see oracle/bee_oracle.c)."""

    def __init__(self):
        self.lib = ctypes.CDLL(str(build_oracle()))
        L = self.lib
        L.oracle_cast_f32_bf16.argtypes = [_vp, _vp, _i64]
        L.oracle_cast_bf16_f32.argtypes = [_vp, _vp, _i64]
        L.oracle_matmul_f32.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64]
        L.oracle_bmm_bf16.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i, _f]
        L.oracle_reduce_rows_f32.argtypes = [_i, _vp, _vp, _i64, _i64]
        L.oracle_reduce_global_i32.argtypes = [_i, _vp, _i64]
        L.oracle_reduce_global_i32.restype = ctypes.c_int32
        L.oracle_sum_f32.argtypes = [_vp, _i64]
        L.oracle_sum_f32.restype = _f
        L.oracle_softmax_f32.argtypes = [_vp, _vp, _i64, _i64]
        L.oracle_rms_norm_f32.argtypes = [_vp, _vp, _vp, _i64, _i64, _f]
        L.oracle_rope_f32.argtypes = [_vp, _vp, _i64, _i64, _i64, _i64, _d, _i64]
        L.oracle_attention_f32.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _f, _vp]

    # elementwise: plain IEEE fp32 / integer arithmetic, as
    # cpu_binary_linear_parallel (Bee/Tensor/Cpu/ElementWiseCpu.hpp:601-625)
    @staticmethod
    def binary(op: int, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        with np.errstate(all="ignore"):
            if op == 0:
                return (a + b).astype(a.dtype)
            if op == 1:
                return (a - b).astype(a.dtype)
            if op == 2:
                return (a * b).astype(a.dtype)
            if np.issubdtype(a.dtype, np.integer):
                return np.trunc(a.astype(np.float64) / b).astype(a.dtype)
            return (a / b).astype(a.dtype)

    def cast_f32_bf16(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(x.shape, np.uint16)
        self.lib.oracle_cast_f32_bf16(_p(x), _p(y), x.size)
        return y

    def matmul_f32(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        m, k = a.shape
        n = b.shape[1]
        c = np.empty((m, n), np.float32)
        self.lib.oracle_matmul_f32(_p(a), _p(b), _p(c), m, k, n)
        return c

    def bmm_bf16(self, a_bits: np.ndarray, b_bits: np.ndarray, b_trans: bool = False, alpha: float = 1.0) -> np.ndarray:
        """a_bits [batch, M, K], b_bits [batch, K, N] (or [batch, N, K] if b_trans), uint16 bf16 bits."""
        a = np.ascontiguousarray(a_bits, np.uint16)
        b = np.ascontiguousarray(b_bits, np.uint16)
        if a.ndim == 2:
            a, b = a[None], b[None]
        batch, m, k = a.shape
        n = b.shape[1] if b_trans else b.shape[2]
        c = np.empty((batch, m, n), np.float32)
        self.lib.oracle_bmm_bf16(_p(a), _p(b), _p(c), batch, m, k, n, int(b_trans), float(alpha))
        return c

    def reduce_rows_f32(self, op: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.shape[0], np.float32)
        self.lib.oracle_reduce_rows_f32(op, _p(x), _p(out), x.shape[0], x.shape[1])
        return out

    def reduce_global_i32(self, op: int, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, np.int32)
        return int(self.lib.oracle_reduce_global_i32(op, _p(x), x.size))

    def sum_f32(self, x: np.ndarray) -> float:
        x = np.ascontiguousarray(x, np.float32)
        return float(self.lib.oracle_sum_f32(_p(x), x.size))

    def softmax_f32(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.lib.oracle_softmax_f32(_p(x), _p(y), x.shape[0], x.shape[1])
        return y

    def rms_norm_f32(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        y = np.empty_like(x)
        self.lib.oracle_rms_norm_f32(_p(x), _p(w), _p(y), x.shape[0], x.shape[1], eps)
        return y

    def rope_f32(self, x: np.ndarray, seq: int, heads: int, hd: int, theta: float = 10000.0,
                 pos_offset: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        rows = x.size // (heads * hd)
        self.lib.oracle_rope_f32(_p(x), _p(y), rows, seq, heads, hd, theta, pos_offset)
        return y

    def attention_f32(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
        q, k, v = (np.ascontiguousarray(t, np.float32) for t in (q, k, v))
        heads, seq, hd = q.shape
        o = np.empty_like(q)
        work = np.empty((seq, seq), np.float32)
        self.lib.oracle_attention_f32(_p(q), _p(k), _p(v), _p(o), heads, seq, hd, scale, _p(work))
        return o

    @staticmethod
    def mean_int(x: np.ndarray, axis=None) -> np.ndarray:
        """Integer mean as the reference computes it (Bee/Tensor/Cpu/ReduceCpu.hpp:431-466,
        551-610): accumulate in double, divide by the count, F64 out.  The
        accumulation is done exactly (int64, or Python integers where int64
        could overflow) and rounded once, which equals the reference's
        sequential double sum whenever that sum is exact (every partial sum
        below 2^53 in magnitude)."""
        x = np.asarray(x)
        n = x.size if axis is None else x.shape[axis]
        bound = int(np.abs(x.astype(np.float64)).max(initial=0.0)) * max(n, 1)
        if bound < 2 ** 62:
            s = x.astype(np.int64).sum(axis=axis, dtype=np.int64)
            return np.asarray(s, np.int64).astype(np.float64) / np.float64(n)
        s = x.astype(object).sum(axis=axis)
        return np.vectorize(lambda v: float(int(v)) / n, otypes=[np.float64])(s)

    @staticmethod
    def strided_gather(flat: np.ndarray, offset: int, shape, strides) -> np.ndarray:
        """Row-major materialisation of the view (offset, shape, strides in
        elements) of the 1-D buffer `flat`: out[i0, .., ik] = flat[offset +
        sum_d i_d * strides[d]] — the stride loop of the reference's
        contiguous_copy_into (Bee/Tensor/Core/Tensor.cpp:119-147), as numpy
        index arithmetic."""
        flat = np.asarray(flat).reshape(-1)
        idx = np.full(tuple(shape), offset, dtype=np.int64)
        for d, (n, st) in enumerate(zip(shape, strides)):
            sh = [1] * len(shape)
            sh[d] = n
            idx = idx + (np.arange(n, dtype=np.int64) * st).reshape(sh)
        return flat[idx]


class Reference:
    """The reference's own CPU path (oracle/_ref/libbee_ref.so, built from its sources)."""

    def __init__(self):
        if not REF_SO.exists():
            raise FileNotFoundError(f"reference CPU library not built: {REF_SO}")
        self.lib = ctypes.CDLL(str(REF_SO))
        L = self.lib
        L.bref_threads.restype = _i
        L.bref_isa.restype = ctypes.c_char_p
        for name, args in {
            "bref_matmul_f32": [_vp, _vp, _vp, _i64, _i64, _i64, _i],
            "bref_binary_f32": [_i, _vp, _vp, _vp, _i64, _i64, _i],
            "bref_reduce_rows_f32": [_i, _vp, _vp, _i64, _i64, _i],
            "bref_reduce_global_i32": [_i, _vp, _i64, _vp, _i],
            "bref_reduce_global_f32": [_i, _vp, _i64, _vp, _i],
            "bref_softmax_f32": [_vp, _vp, _i64, _i64, _i],
            "bref_rms_norm_f32": [_vp, _vp, _vp, _i64, _i64, _f, _i],
            "bref_rope_f32": [_vp, _vp, _i64, _i64, _i64, _i64, _d, _i64, _i],
            "bref_attention_f32": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _f, _i],
            "bref_view_copy_f32": [_vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i],
            "bref_binary_bcast_f32": [_i, _vp, _vp, _vp, _vp, _i, _vp, _i],
            "bref_mean_int": [_i, _vp, _i64, _i64, _i64, _i, _vp, _i],
            "bref_sweep": [_vp, _vp, _vp, _i64, _i64, _vp],
        }.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _d

    @staticmethod
    def _chk(t: float, what: str) -> float:
        if t < 0:
            raise RuntimeError(f"reference {what} failed")
        return t

    def threads(self) -> int:
        return int(self.lib.bref_threads())

    def sweep(self, x, y, xi):
        """One timed step of the memory-bound sweep (add, mul, row sum, row max,
        row softmax, int32 sum) on the reference's CPU path; the arrays must stay
        alive between calls (their Tensors are cached by address)."""
        rows, cols = x.shape
        t = np.zeros(6, np.float64)
        tot = self._chk(self.lib.bref_sweep(_p(x), _p(y), _p(xi), rows, cols, _p(t)), "sweep")
        names = ["add_f32", "mul_f32", "row_sum_f32", "row_max_f32", "softmax_f32", "sum_i32"]
        return tot, dict(zip(names, map(float, t)))

    def isa(self) -> str:
        """bee::simd::isa_name(bee::simd::current_isa()) on this host."""
        return self.lib.bref_isa().decode()

    def matmul_f32(self, a, b, reps=1):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        c = np.empty((a.shape[0], b.shape[1]), np.float32)
        t = self._chk(self.lib.bref_matmul_f32(_p(a), _p(b), _p(c), a.shape[0], a.shape[1], b.shape[1], reps), "matmul")
        return c, t

    def binary_f32(self, op, a, b, reps=1):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.empty_like(a)
        a2 = a.reshape(a.shape[0], -1) if a.ndim > 1 else a.reshape(1, -1)
        t = self._chk(self.lib.bref_binary_f32(op, _p(a), _p(b), _p(out), a2.shape[0], a2.shape[1], reps), "binary")
        return out, t

    def reduce_rows_f32(self, op, x, reps=1):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.shape[0], np.float32)
        t = self._chk(self.lib.bref_reduce_rows_f32(op, _p(x), _p(out), x.shape[0], x.shape[1], reps), "reduce rows")
        return out, t

    def reduce_global_i32(self, op, x, reps=1):
        x = np.ascontiguousarray(x, np.int32)
        out = np.zeros(1, np.int32)
        t = self._chk(self.lib.bref_reduce_global_i32(op, _p(x), x.size, _p(out), reps), "reduce global")
        return int(out[0]), t

    def reduce_global_f32(self, op, x, reps=1):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(1, np.float32)
        t = self._chk(self.lib.bref_reduce_global_f32(op, _p(x), x.size, _p(out), reps), "reduce global")
        return float(out[0]), t

    def softmax_f32(self, x, reps=1):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        t = self._chk(self.lib.bref_softmax_f32(_p(x), _p(y), x.shape[0], x.shape[1], reps), "softmax")
        return y, t

    def rms_norm_f32(self, x, w, eps, reps=1):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        y = np.empty_like(x)
        t = self._chk(self.lib.bref_rms_norm_f32(_p(x), _p(w), _p(y), x.shape[0], x.shape[1], eps, reps), "rms_norm")
        return y, t

    def rope_f32(self, x, seq, heads, hd, theta=10000.0, pos_offset=0, reps=1):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        rows = x.size // (heads * hd)
        t = self._chk(self.lib.bref_rope_f32(_p(x), _p(y), rows, seq, heads, hd, theta, pos_offset, reps), "rope")
        return y, t

    def attention_f32(self, q, k, v, scale, reps=1):
        q, k, v = (np.ascontiguousarray(t, np.float32) for t in (q, k, v))
        o = np.empty_like(q)
        heads, seq, hd = q.shape
        t = self._chk(self.lib.bref_attention_f32(_p(q), _p(k), _p(v), _p(o), heads, seq, hd, scale, reps), "attention")
        return o, t


    def binary_bcast_f32(self, op, a, b, reps=1):
        """a op b with broadcasting (equal ranks), on the reference's CPU path."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.empty(np.broadcast_shapes(a.shape, b.shape), np.float32)
        ash = np.array(a.shape, np.int64)
        bsh = np.array(b.shape, np.int64)
        t = self._chk(self.lib.bref_binary_bcast_f32(op, _p(a), _p(ash), _p(b), _p(bsh), a.ndim, _p(out), reps),
                      "binary broadcast")
        return out, t

    def mean_int(self, x, global_mean=False, reps=1):
        """Mean over dim 1 of the [outer, axis, inner] integer tensor x (or of
        all elements), F64 result, on the reference's CPU path."""
        dt = 2 if x.dtype == np.int32 else 3
        x = np.ascontiguousarray(x)
        o, a, i = x.shape
        out = np.empty(1 if global_mean else o * i, np.float64)
        t = self._chk(self.lib.bref_mean_int(dt, _p(x), o, a, i, int(global_mean), _p(out), reps), "mean")
        return (out[0] if global_mean else out.reshape(o, i)), t

    def view_copy_f32(self, x, perm, slices=None, reps=1):
        """permute(perm), then slice(d, start, end, step) per dim of `slices`
        (None = whole dim), then contiguous(), on the reference's CPU path."""
        x = np.ascontiguousarray(x, np.float32)
        nd = x.ndim
        shape = np.array(x.shape, np.int64)
        permv = np.array(perm, np.int32)
        st = np.zeros(nd, np.int64)
        en = np.zeros(nd, np.int64)
        sp = np.zeros(nd, np.int64)
        out_shape = [x.shape[p] for p in perm]
        for d, sl in enumerate(slices or [None] * nd):
            if sl is None:
                continue
            st[d], en[d], sp[d] = sl
            out_shape[d] = len(range(sl[0], sl[1], sl[2]))
        out = np.empty(out_shape, np.float32)
        t = self._chk(self.lib.bref_view_copy_f32(_p(x), nd, _p(shape), _p(permv), _p(st), _p(en), _p(sp), _p(out),
                                                  reps), "view_copy")
        return out, t


def reference_available() -> bool:
    return REF_SO.exists()
