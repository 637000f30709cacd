"""Mirror of tv/quantization/engine.tkv (PTQ calibration + INT8 quantize).

Same names, argument order and errors as the reference; buffers are numpy
arrays (host, the reference's lists -- int8 or int32 element type) or torch
CUDA tensors (device, asynchronous on the current stream).  All arithmetic
runs in libtvq's CUDA kernels.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .. import _native as N
from . import _buf as B
from .types import QuantParams, identity

__all__ = ["calibrate_minmax", "calibrate_minmax_batches", "calibrate_per_channel_minmax",
           "quantize_int8_symmetric", "dequantize_int8_symmetric", "quantize_int8_per_channel",
           "dequantize_int8_per_channel", "quantize_dynamic_int8_rowwise"]


def _params(scale, zp, mn, mx) -> QuantParams:
    return QuantParams(scale.value, zp.value, mn.value, mx.value)


def calibrate_minmax(data, symmetric: int = 1) -> QuantParams:
    """calibrate_minmax, engine.tkv:13-36"""
    return calibrate_minmax_batches([data], symmetric)


def calibrate_minmax_batches(batches, symmetric: int = 1) -> QuantParams:
    """calibrate_minmax over the concatenation of several batches (running
    min/max on the GPU), as BASELINE config 1 calibrates over 8 batches."""
    arrs = [B.host_f32(b).ravel() for b in batches]
    if sum(a.size for a in arrs) == 0:
        return identity()
    ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    sizes = (C.c_int64 * len(arrs))(*[a.size for a in arrs])
    s, zp, mn, mx = C.c_float(), C.c_int64(), C.c_float(), C.c_float()
    N.call("tvq_calibrate_minmax_batches", ptrs, sizes, len(arrs), int(symmetric), C.byref(s), C.byref(zp),
           C.byref(mn), C.byref(mx))
    return _params(s, zp, mn, mx)


def calibrate_per_channel_minmax(data, rows: int, cols: int, symmetric: int = 1) -> list:
    """calibrate_per_channel_minmax, engine.tkv:202-213"""
    if rows <= 0 or cols <= 0:
        raise ValueError("rows/cols must be > 0")
    d = B.host_f32(data).ravel()
    if d.size < rows * cols:
        raise ValueError("data smaller than rows*cols")
    sc = np.empty(rows, np.float32)
    zp = np.empty(rows, np.int64)
    mn = np.empty(rows, np.float32)
    mx = np.empty(rows, np.float32)
    N.call("tvq_calibrate_per_channel_params", B.ptr(d), d.size, rows, cols, int(bool(symmetric)), B.ptr(sc),
           B.ptr(zp), B.ptr(mn), B.ptr(mx), rows)
    return [QuantParams(float(sc[r]), int(zp[r]), float(mn[r]), float(mx[r])) for r in range(rows)]


def _i8_dst(dst):
    """(device-or-host int8 target, int32 host list or None)."""
    if B.is_dev(dst):
        return dst, None
    if dst.dtype == np.int8:
        return dst, None
    if dst.dtype == np.int32:  # the reference's list[i32] storage
        return np.empty(dst.shape, np.int8), dst
    raise TypeError("dst must be int8 or int32")


def quantize_int8_symmetric(src, dst, scale: float) -> int:
    """quantize_int8_symmetric, engine.tkv:216-226"""
    if B.size(dst) < B.size(src):
        raise ValueError("dst too small")
    if B.is_dev(src):
        import torch
        sdev = torch.tensor([scale], dtype=torch.float32, device=src.device)
        N.call("tvq_dev_quantize_int8", B.ptr(src), B.ptr(dst), src.numel(), B.ptr(sdev), B.stream_of(src))
        return 0
    s = B.host_f32(src).ravel()
    tgt, wide = _i8_dst(dst)
    N.call("tvq_quantize_int8_symmetric", B.ptr(s), s.size, B.ptr(tgt), tgt.size, float(scale))
    if wide is not None:
        wide.ravel()[:s.size] = tgt.ravel()[:s.size]
    return 0


def dequantize_int8_symmetric(src, dst, scale: float) -> int:
    """dequantize_int8_symmetric, engine.tkv:229-234"""
    if B.size(dst) < B.size(src):
        raise ValueError("dst too small")
    q = np.ascontiguousarray(np.asarray(src), dtype=np.int8)
    out = np.empty(q.shape, np.float32)
    N.call("tvq_dequantize_int8_symmetric", B.ptr(q), q.size, B.ptr(out), out.size, float(scale))
    np.asarray(dst).ravel()[:q.size] = out.ravel()
    return 0


def quantize_int8_per_channel(src, dst, rows: int, cols: int, scales) -> int:
    """quantize_int8_per_channel, engine.tkv:237-250"""
    if B.size(dst) < rows * cols or B.size(src) < rows * cols:
        raise ValueError("span too small")
    if B.size(scales) < rows:
        raise ValueError("scales smaller than rows")
    if B.is_dev(src):
        N.call("tvq_dev_quantize_int8_per_channel", B.ptr(src), B.ptr(dst), B.ptr(scales), rows, cols,
               B.stream_of(src))
        return 0
    s = B.host_f32(src).ravel()
    sc = B.host_f32(scales).ravel()
    tgt, wide = _i8_dst(dst)
    N.call("tvq_quantize_int8_per_channel", B.ptr(s), s.size, B.ptr(tgt), tgt.size, rows, cols, B.ptr(sc), sc.size)
    if wide is not None:
        wide.ravel()[:rows * cols] = tgt.ravel()[:rows * cols]
    return 0


def dequantize_int8_per_channel(src, dst, rows: int, cols: int, scales) -> int:
    """dequantize_int8_per_channel, engine.tkv:253-262"""
    if B.size(dst) < rows * cols or B.size(src) < rows * cols:
        raise ValueError("span too small")
    if B.size(scales) < rows:
        raise ValueError("scales smaller than rows")
    q = np.ascontiguousarray(np.asarray(src), dtype=np.int8).ravel()
    sc = B.host_f32(scales).ravel()
    out = np.empty(q.size, np.float32)
    N.call("tvq_dequantize_int8_per_channel", B.ptr(q), q.size, B.ptr(out), out.size, rows, cols, B.ptr(sc), sc.size)
    np.asarray(dst).ravel()[:rows * cols] = out[:rows * cols]
    return 0


def quantize_dynamic_int8_rowwise(src, dst, rows: int, cols: int, scales_out) -> int:
    """quantize_dynamic_int8_rowwise, engine.tkv:266-285"""
    if B.size(dst) < rows * cols or B.size(src) < rows * cols:
        raise ValueError("span too small")
    if B.size(scales_out) < rows:
        raise ValueError("scales_out smaller than rows")
    if B.is_dev(src):
        N.call("tvq_dev_quantize_dynamic_rowwise", B.ptr(src), B.ptr(dst), B.ptr(scales_out), rows, cols,
               B.stream_of(src))
        return 0
    s = B.host_f32(src).ravel()
    tgt, wide = _i8_dst(dst)
    so = np.empty(rows, np.float32)
    N.call("tvq_quantize_dynamic_int8_rowwise", B.ptr(s), s.size, B.ptr(tgt), tgt.size, rows, cols, B.ptr(so), rows)
    np.asarray(scales_out).ravel()[:rows] = so
    if wide is not None:
        wide.ravel()[:rows * cols] = tgt.ravel()[:rows * cols]
    return 0
