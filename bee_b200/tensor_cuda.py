"""Python mirror of ``bee::tensor::cuda`` (Bee/Tensor/Cuda/Backend.hpp:20-84).

Same operation names and argument meaning as the reference's host bridge, over
torch CUDA tensors (torch supplies device memory and the stream; every kernel is
ours, reached through the C ABI).  Like the reference bridge each call is
synchronous from the caller's point of view only if ``sync=True``; by default
work is enqueued on torch's current stream and ordered with other torch work.
Errors raise ``BeeError`` carrying the status and message; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _capi as C
from ._capi import BeeError  # noqa: F401  (re-export)

DTYPE_CODE = {
    torch.bool: C.BOOL, torch.uint8: C.U8, torch.int32: C.I32, torch.int64: C.I64,
    torch.float32: C.F32, torch.float64: C.F64, torch.int8: C.I8, torch.float16: C.F16,
    torch.bfloat16: C.BF16,
}


def _code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise BeeError("dtype", 1, f"unsupported torch dtype {t.dtype}") from None


def _dev(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise BeeError("device", 1, "tensor is not on a CUDA device")
        if not t.is_contiguous():
            raise BeeError("layout", 1, "tensor is not contiguous")


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _done(sync: bool, stream=None) -> None:
    if sync:
        C.call("bee_b200_stream_synchronize", _stream(stream))


def ew_binary(op: int, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *, stream=None, sync=False):
    """out = a (op) b elementwise (tensor::cuda::ew_binary, Backend.hpp:51)."""
    _dev(a, b, out)
    if not (a.dtype == b.dtype == out.dtype) or not (a.numel() == b.numel() == out.numel()):
        raise BeeError("ew_binary", 1, "a, b, out must share dtype and element count")
    C.call("bee_b200_ew_binary", op, _code(a), a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _stream(stream))
    _done(sync, stream)
    return out


def ew_unary(op: int, src: torch.Tensor, dst: torch.Tensor, *, stream=None, sync=False):
    """dst = op(src) (tensor::cuda::ew_unary, Backend.hpp:54)."""
    _dev(src, dst)
    C.call("bee_b200_ew_unary", op, _code(src), src.data_ptr(), dst.data_ptr(), src.numel(), _stream(stream))
    _done(sync, stream)
    return dst


def ew_cast(src: torch.Tensor, dst: torch.Tensor, *, stream=None, sync=False):
    """dst = cast(src) (tensor::cuda::ew_cast, Backend.hpp:57), incl. fp32 -> bf16."""
    _dev(src, dst)
    if src.numel() != dst.numel():
        raise BeeError("ew_cast", 1, "element counts differ")
    C.call("bee_b200_ew_cast", _code(src), src.data_ptr(), _code(dst), dst.data_ptr(), src.numel(), _stream(stream))
    _done(sync, stream)
    return dst


def scale_fp(buf: torch.Tensor, factor: float, *, stream=None, sync=False):
    """buf *= factor (tensor::cuda::scale_fp, Backend.hpp:66)."""
    _dev(buf)
    C.call("bee_b200_scale_fp", _code(buf), buf.data_ptr(), float(factor), buf.numel(), _stream(stream))
    _done(sync, stream)
    return buf


def reduce_global(op: int, src: torch.Tensor, dst: torch.Tensor, *, stream=None, sync=False):
    """dst[0] = reduce(src) (tensor::cuda::reduce_global, Backend.hpp:60)."""
    _dev(src, dst)
    C.call("bee_b200_reduce_global", op, _code(src), src.data_ptr(), dst.data_ptr(), src.numel(), _stream(stream))
    _done(sync, stream)
    return dst


def reduce_axis(op: int, src: torch.Tensor, dst: torch.Tensor, outer: int, axis: int, inner: int, *, stream=None,
                sync=False):
    """[outer, axis, inner] -> [outer, inner] (tensor::cuda::reduce_axis, Backend.hpp:63)."""
    _dev(src, dst)
    C.call("bee_b200_reduce_axis", op, _code(src), src.data_ptr(), dst.data_ptr(), outer, axis, inner,
           _stream(stream))
    _done(sync, stream)
    return dst


def softmax_rows(src: torch.Tensor, dst: torch.Tensor, *, stream=None, sync=False):
    """Row softmax of a [rows, cols] tensor (last dim)."""
    _dev(src, dst)
    cols = src.shape[-1]
    rows = src.numel() // cols if cols else 0
    C.call("bee_b200_softmax_rows", _code(src), src.data_ptr(), dst.data_ptr(), rows, cols, _stream(stream))
    _done(sync, stream)
    return dst


def rms_norm_rows(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, eps: float = 1e-6, *, stream=None, sync=False):
    """y = x / sqrt(mean(x^2) + eps) * w over the last dim."""
    _dev(x, w, y)
    cols = x.shape[-1]
    C.call("bee_b200_rms_norm_rows", _code(x), x.data_ptr(), w.data_ptr(), y.data_ptr(), x.numel() // cols, cols,
           float(eps), _stream(stream))
    _done(sync, stream)
    return y


def rope(x: torch.Tensor, y: torch.Tensor, seq: int, heads: int, head_dim: int, theta: float = 10000.0,
         pos_offset: int = 0, *, stream=None, sync=False):
    """Rotate-half RoPE on x viewed [rows, heads, head_dim], position = row % seq + pos_offset."""
    _dev(x, y)
    rows = x.numel() // (heads * head_dim)
    C.call("bee_b200_rope", _code(x), x.data_ptr(), y.data_ptr(), rows, seq, heads, head_dim, float(theta),
           pos_offset, _stream(stream))
    _done(sync, stream)
    return y


def rms_norm_rope(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, seq: int, heads: int, head_dim: int,
                  eps: float = 1e-6, theta: float = 10000.0, pos_offset: int = 0, *, stream=None, sync=False):
    """RMSNorm then RoPE in one pass over [rows, heads*head_dim]."""
    _dev(x, w, y)
    rows = x.numel() // (heads * head_dim)
    C.call("bee_b200_rms_norm_rope", _code(x), x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, seq, heads, head_dim,
           float(eps), float(theta), pos_offset, _stream(stream))
    _done(sync, stream)
    return y
