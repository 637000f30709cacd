"""Mirror of tv/quantization/int4.tkv: group-wise INT4 weights (GPTQ / AWQ
layout) on the B200.

Weights [rows, cols] -> packed bytes [rows, cols/2] (two nibbles per byte,
low nibble first, biased by +8 in the symmetric form) + per-group scales
[rows, cols/group_size] (+ zero points in the asymmetric form).  The
reference fills caller-provided lists (packed_out, scales_out, zps_out);
here the out arguments are numpy arrays or torch CUDA tensors written in
place, or omitted and returned.  ValueError where the reference raises.
Codecs are bit-exact with the reference; matmul_int4_grouped runs on the
tensor cores (fp32 activations split into fp16 hi / lo, the weights'
integers exact in fp16, each group's partial sum times its scale).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .. import _native as N
from . import _buf as B

__all__ = ["quantize_int4_grouped", "dequantize_int4_grouped", "quantize_int4_grouped_asym",
           "dequantize_int4_grouped_asym", "permute_cols", "inv_permute_cols", "matmul_int4_grouped",
           "matmul_int4_grouped_ordered"]


def _check_shape(cols: int, group_size: int):
    if group_size <= 0 or cols % group_size != 0:
        raise ValueError("cols must be a multiple of group_size")
    if cols % 2 != 0:
        raise ValueError("cols must be even for nibble packing")


def _quantize(src, rows, cols, group_size, packed_out, scales_out, zps_out, asym):
    _check_shape(cols, group_size)
    ng = cols // group_size
    if B.is_dev(src):
        import torch
        dev = src.device
        packed = packed_out if packed_out is not None else torch.empty(rows * cols // 2, dtype=torch.uint8, device=dev)
        scales = scales_out if scales_out is not None else torch.empty(rows * ng, dtype=torch.float32, device=dev)
        zps = (zps_out if zps_out is not None else torch.empty(rows * ng, dtype=torch.int64, device=dev)) if asym \
            else None
        N.call("tvq_dev_quantize_int4_grouped", B.ptr(src), rows, cols, group_size, B.ptr(packed), B.ptr(scales),
               B.ptr(zps), B.stream_of(src))
        return (packed, scales, zps) if asym else (packed, scales)
    x = B.host_f32(src).ravel()
    if x.size < rows * cols:
        raise ValueError("src smaller than rows*cols")
    packed = np.zeros(rows * cols // 2, np.uint8)
    scales = np.zeros(rows * ng, np.float32)
    zps = np.zeros(rows * ng, np.int64) if asym else None
    N.call("tvq_quantize_int4_grouped", B.ptr(x), rows, cols, group_size, B.ptr(packed), B.ptr(scales), B.ptr(zps))
    if packed_out is not None:
        if B.size(packed_out) < rows * cols // 2:
            raise ValueError("packed_out too small")
        np.asarray(packed_out).reshape(-1)[:packed.size] = packed
    if scales_out is not None:
        np.asarray(scales_out).reshape(-1)[:scales.size] = scales
    if asym and zps_out is not None:
        np.asarray(zps_out).reshape(-1)[:zps.size] = zps
    return (packed, scales, zps) if asym else (packed, scales)


def quantize_int4_grouped(src, rows: int, cols: int, group_size: int, packed_out=None, scales_out=None):
    """quantize_int4_grouped, int4.tkv:27-48 -> (packed, scales)."""
    return _quantize(src, rows, cols, group_size, packed_out, scales_out, None, False)


def quantize_int4_grouped_asym(src, rows: int, cols: int, group_size: int, packed_out=None, scales_out=None,
                               zps_out=None):
    """quantize_int4_grouped_asym, int4.tkv:68-150 -> (packed, scales, zps)."""
    return _quantize(src, rows, cols, group_size, packed_out, scales_out, zps_out, True)


def _dequantize(packed, dst, rows, cols, group_size, scales, zps):
    _check_shape(cols, group_size)
    ng = cols // group_size
    if B.size(scales) < rows * ng:
        raise ValueError("scales smaller than rows*num_groups")
    if B.is_dev(packed):
        import torch
        out = dst if dst is not None else torch.empty(rows * cols, dtype=torch.float32, device=packed.device)
        N.call("tvq_dev_dequantize_int4_grouped", B.ptr(packed), B.ptr(out), rows, cols, group_size, B.ptr(scales),
               B.ptr(zps), B.stream_of(packed))
        return out
    pk = np.ascontiguousarray(np.asarray(packed).astype(np.int64).astype(np.uint8)).ravel()
    sc = B.host_f32(scales).ravel()
    zp = np.ascontiguousarray(np.asarray(zps, np.int64)).ravel() if zps is not None else None
    out = np.empty(rows * cols, np.float32)
    N.call("tvq_dequantize_int4_grouped", B.ptr(pk), B.ptr(out), rows, cols, group_size, B.ptr(sc), sc.size,
           B.ptr(zp))
    if dst is not None:
        if B.size(dst) < rows * cols:
            raise ValueError("dst too small")
        np.asarray(dst).reshape(-1)[:out.size] = out
        return dst
    return out


def dequantize_int4_grouped(packed, dst, rows: int, cols: int, group_size: int, scales):
    """dequantize_int4_grouped, int4.tkv:51-64 (dst may be None: returned)."""
    return _dequantize(packed, dst, rows, cols, group_size, scales, None)


def dequantize_int4_grouped_asym(packed, dst, rows: int, cols: int, group_size: int, scales, zps):
    """dequantize_int4_grouped_asym, int4.tkv:153-164."""
    return _dequantize(packed, dst, rows, cols, group_size, scales, zps)


def _permute(src, rows, cols, perm, inverse):
    if B.size(perm) != cols:
        raise ValueError("perm length must equal cols")
    if B.is_dev(src):
        import torch
        out = torch.zeros(rows * cols, dtype=torch.float32, device=src.device)
        N.call("tvq_dev_permute_cols", B.ptr(src), B.ptr(out), rows, cols, B.ptr(perm), 1 if inverse else 0,
               B.stream_of(src))
        return out
    x = B.host_f32(src).ravel()
    pm = np.ascontiguousarray(np.asarray(perm, np.int64)).ravel()
    out = np.empty(rows * cols, np.float32)
    N.call("tvq_permute_cols", B.ptr(x), B.ptr(out), rows, cols, B.ptr(pm), pm.size, 1 if inverse else 0)
    return out


def permute_cols(src, rows: int, cols: int, perm):
    """permute_cols, int4.tkv:169-175: out[r, c] = src[r, perm[c]]."""
    return _permute(src, rows, cols, perm, False)


def inv_permute_cols(src, rows: int, cols: int, perm):
    """inv_permute_cols, int4.tkv:178-184: out[r, perm[c]] = src[r, c]."""
    return _permute(src, rows, cols, perm, True)


def _matmul(pa, packed_w, pbias, py, m, n, k, group_size, scales_w, perm):
    if group_size <= 0 or k % group_size != 0 or k % 2 != 0:
        raise ValueError("k must be an even multiple of group_size")
    ng = k // group_size
    if B.size(scales_w) < n * ng:
        raise ValueError("scales_w smaller than N*num_groups")
    nb = B.size(pbias)
    if B.is_dev(pa):
        N.call("tvq_dev_matmul_int4_grouped", B.ptr(pa), B.ptr(packed_w), B.ptr(pbias) if nb else None, B.ptr(py),
               m, n, k, group_size, B.ptr(scales_w), B.ptr(perm) if perm is not None else None, B.stream_of(pa))
        return 0
    A = B.host_f32(pa).ravel()
    pk = np.ascontiguousarray(np.asarray(packed_w).astype(np.int64).astype(np.uint8)).ravel()
    sc = B.host_f32(scales_w).ravel()
    bias = B.host_f32(pbias).ravel() if nb else None
    pm = np.ascontiguousarray(np.asarray(perm, np.int64)).ravel() if perm is not None else None
    Y = np.empty(m * n, np.float32)
    N.call("tvq_matmul_int4_grouped", B.ptr(A), B.ptr(pk), B.ptr(bias), nb, B.ptr(Y), m, n, k, group_size,
           B.ptr(sc), sc.size, B.ptr(pm))
    np.asarray(py).reshape(-1)[:m * n] = Y
    return 0


def matmul_int4_grouped(pa, packed_w, pbias, py, m: int, n: int, k: int, group_size: int, scales_w) -> int:
    """matmul_int4_grouped, int4.tkv:213-239: py = pa @ dequant(packed_w)^T + pbias."""
    return _matmul(pa, packed_w, pbias, py, m, n, k, group_size, scales_w, None)


def matmul_int4_grouped_ordered(pa, packed_w, pbias, py, m: int, n: int, k: int, group_size: int, scales_w,
                                perm) -> int:
    """matmul_int4_grouped_ordered (GPTQ act-order), int4.tkv:187-208: the
    activation columns gathered by perm inside the GEMM."""
    if B.size(perm) != k:
        raise ValueError("perm length must equal k")
    return _matmul(pa, packed_w, pbias, py, m, n, k, group_size, scales_w, perm)
