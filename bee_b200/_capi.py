"""ctypes binding of the C ABI in ``include/bee_b200.h``.

The library is the in-tree ``bee_b200/_lib/libbee_b200.so`` built by
``bee_b200.build``.  There is no fallback: if the library is missing or fails
to load, every call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libbee_b200.so"

# dtype codes (bee::DType, Bee/Tensor/Core/DType.hpp:17-32)
BOOL, U8, I32, I64, F32, F64, I8, F16, BF16 = range(9)
# op codes (Bee/CUDA/Api.hpp:77-100)
ADD, SUB, MUL, DIV = range(4)
NEG, ABS, SQRT, EXP, LOG = range(5)
SUM, MIN, MAX, PROD = range(4)


class BeeError(RuntimeError):
    """A bee_b200 call returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status}: {message}")
        self.status = status
        self.message = message


_c = ctypes
_vp, _sz, _i, _f, _d = _c.c_void_p, _c.c_size_t, _c.c_int, _c.c_float, _c.c_double

# name -> argtypes (restype int unless listed in _RESTYPES)
SIGNATURES = {
    "bee_b200_last_error": [],
    "bee_b200_status_string": [_i],
    "bee_b200_version": [],
    "bee_b200_allocate": [_c.POINTER(_vp), _sz, _sz, _vp],
    "bee_b200_deallocate": [_vp, _vp],
    "bee_b200_memcpy_h2d": [_vp, _vp, _sz, _vp],
    "bee_b200_memcpy_d2h": [_vp, _vp, _sz, _vp],
    "bee_b200_memcpy_d2d": [_vp, _vp, _sz, _vp],
    "bee_b200_memset": [_vp, _i, _sz, _vp],
    "bee_b200_stream_synchronize": [_vp],
    "bee_b200_clock_probe": [_c.c_ulonglong, _vp, _vp],
    "bee_b200_set_device": [_i],
    "bee_b200_get_device": [_c.POINTER(_i)],
    "bee_b200_device_count": [_c.POINTER(_i)],
    "bee_b200_ew_binary": [_i, _i, _vp, _vp, _vp, _sz, _vp],
    "bee_b200_ew_binary_strided": [_i, _i, _i, _c.POINTER(_c.c_int64), _vp, _c.POINTER(_c.c_int64), _vp,
                                   _c.POINTER(_c.c_int64), _vp, _vp],
    "bee_b200_ew_unary": [_i, _i, _vp, _vp, _sz, _vp],
    "bee_b200_ew_cast": [_i, _vp, _i, _vp, _sz, _vp],
    "bee_b200_scale_fp": [_i, _vp, _d, _sz, _vp],
    "bee_b200_reduce_global": [_i, _i, _vp, _vp, _sz, _vp],
    "bee_b200_reduce_global_noalloc": [_i, _i, _vp, _vp, _sz, _vp],
    "bee_b200_reduce_global_allranks": [_i, _i, _vp, _sz, _vp, _c.POINTER(_vp), _i, _i, _c.c_uint,
                                        _c.c_ulonglong, _vp],
    "bee_b200_reduce_axis": [_i, _i, _vp, _vp, _sz, _sz, _sz, _vp],
    "bee_b200_reduce_mean_int": [_i, _vp, _vp, _sz, _sz, _sz, _vp],
    "bee_b200_softmax_rows": [_i, _vp, _vp, _sz, _sz, _vp],
    "bee_b200_softmax_rows_to": [_i, _vp, _i, _vp, _sz, _sz, _vp],
    "bee_b200_rms_norm_rows": [_i, _vp, _vp, _vp, _sz, _sz, _f, _vp],
    "bee_b200_rope": [_i, _vp, _vp, _sz, _sz, _sz, _sz, _d, _sz, _vp],
    "bee_b200_rms_norm_rope": [_i, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _f, _d, _sz, _vp],
    "bee_b200_matmul": [_i, _vp, _vp, _vp, _sz, _sz, _sz, _vp],
    "bee_b200_bmm": [_i, _i, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _i, _f, _vp],
    "bee_b200_bmm_strided": [_i, _i, _vp, _c.c_int64, _c.c_int64, _vp, _c.c_int64, _c.c_int64, _vp, _c.c_int64,
                             _c.c_int64, _sz, _sz, _sz, _sz, _i, _f, _vp],
    "bee_b200_attention": [_i, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _f, _vp],
    "bee_b200_transpose_2d": [_i, _vp, _vp, _sz, _sz, _vp],
    "bee_b200_strided_copy": [_i, _vp, _i, _c.POINTER(_c.c_int64), _c.POINTER(_c.c_int64), _vp, _vp],
    "bee_b200_splitk_recv_bytes": [_sz, _sz, _i],
    "bee_b200_gemm_splitk_scatter": [_vp, _sz, _vp, _sz, _sz, _sz, _c.POINTER(_vp), _i, _i, _vp],
    "bee_b200_gemm_splitk_reduce": [_vp, _c.POINTER(_vp), _sz, _sz, _i, _i, _vp],
    "bee_b200_ipc_alloc": [_c.POINTER(_vp), _sz],
    "bee_b200_ipc_free": [_vp],
    "bee_b200_ipc_handle": [_vp, _vp],
    "bee_b200_ipc_open": [_vp, _c.POINTER(_vp)],
    "bee_b200_ipc_close": [_vp],
    "bee_b200_device_status": [_c.POINTER(_i)],
}
_RESTYPES = {"bee_b200_last_error": _c.c_char_p, "bee_b200_status_string": _c.c_char_p,
             "bee_b200_splitk_recv_bytes": _sz}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """Loads (once) and returns the library; raises if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"bee_b200 CUDA library not built: {LIB_PATH} (run python -m bee_b200.build)")
                h = ctypes.CDLL(str(LIB_PATH))
                for name, args in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPES.get(name, _i)
                _lib = h
    return _lib


def call(name: str, *args) -> None:
    """Calls a status-returning entry point and raises BeeError on failure."""
    h = lib()
    rc = getattr(h, name)(*args)
    if rc != 0:
        msg = h.bee_b200_last_error().decode(errors="replace")
        raise BeeError(name, rc, msg)


def last_error() -> str:
    return lib().bee_b200_last_error().decode(errors="replace")
