"""Mirror of tv/quantization/matmul.tkv (quantized GEMMs + FP8 quantize).

Signatures follow the reference: (pa, pw, pbias, py, m, n, k, ...) with pa
int8 [m,k], pw int8 [n,k], pbias f32 [n] or empty, py f32 [m,n] written in
place; ValueError where the reference raises.  Buffers may be numpy arrays
(int8, or the reference's int32 lists) or torch CUDA tensors.  The GEMM runs
on the B200 tensor cores (tcgen05) through libtvq.
"""
from __future__ import annotations

import numpy as np

from .. import _native as N
from . import _buf as B

__all__ = ["matmul_int8_symmetric", "matmul_int8_per_channel", "matmul_int8_asymmetric", "matmul_fp8_e4m3",
           "matmul_fp16", "quantize_fp16", "quantize_fp8_e4m3", "quantize_fp8_e4m3_scaled", "dequantize_fp8_e4m3",
           "gemm_i8_accumulators"]


def _as_i8(x) -> np.ndarray:
    a = np.asarray(x)
    if a.dtype == np.int8:
        return np.ascontiguousarray(a)
    return np.ascontiguousarray(a.astype(np.int64).astype(np.int8))


def _bias(pbias):
    if pbias is None or B.size(pbias) == 0:
        return None, 0
    return pbias, B.size(pbias)


def _dev_scalar(v, like):
    import torch
    return torch.tensor([float(v)], dtype=torch.float32, device=like.device)


def matmul_int8_per_channel(pa, pw, pbias, py, m: int, n: int, k: int, scale_a: float, scales_w,
                            act: int = N.ACT_NONE) -> int:
    """matmul_int8_per_channel, matmul.tkv:17-29"""
    if B.size(scales_w) < n:
        raise ValueError("scales_w smaller than N")
    bias, nb = _bias(pbias)
    if B.is_dev(pa):
        sa = _dev_scalar(scale_a, pa)
        N.call("tvq_dev_gemm", N.GEMM_I8, B.ptr(pa), B.ptr(pw), B.ptr(bias), None, B.ptr(py), None, m, n, k,
               B.ptr(sa), B.ptr(scales_w), 1, act, None, None, B.stream_of(pa))
        return 0
    A, W = _as_i8(pa), _as_i8(pw)
    bh = B.host_f32(bias) if bias is not None else None
    sw = B.host_f32(scales_w).ravel()
    Y = np.empty(m * n, np.float32)
    N.call("tvq_matmul_int8_per_channel", B.ptr(A), B.ptr(W), B.ptr(bh), nb, B.ptr(Y), m, n, k, float(scale_a),
           B.ptr(sw), sw.size, act)
    np.asarray(py).reshape(-1)[:m * n] = Y
    return 0


def matmul_int8_symmetric(pa, pw, pbias, py, m: int, n: int, k: int, scale_a: float, scale_w: float,
                          act: int = N.ACT_NONE) -> int:
    """matmul_int8_symmetric, matmul.tkv:4-15"""
    bias, nb = _bias(pbias)
    if B.is_dev(pa):
        sa = _dev_scalar(scale_a, pa)
        sw = _dev_scalar(scale_w, pa)
        N.call("tvq_dev_gemm", N.GEMM_I8, B.ptr(pa), B.ptr(pw), B.ptr(bias), None, B.ptr(py), None, m, n, k,
               B.ptr(sa), B.ptr(sw), 0, act, None, None, B.stream_of(pa))
        return 0
    A, W = _as_i8(pa), _as_i8(pw)
    bh = B.host_f32(bias) if bias is not None else None
    Y = np.empty(m * n, np.float32)
    N.call("tvq_matmul_int8_symmetric", B.ptr(A), B.ptr(W), B.ptr(bh), nb, B.ptr(Y), m, n, k, float(scale_a),
           float(scale_w), act)
    np.asarray(py).reshape(-1)[:m * n] = Y
    return 0


def gemm_i8_accumulators(pa, pw, m: int, n: int, k: int) -> np.ndarray:
    """Raw int32 accumulators of the tensor-core GEMM (_dot_int8 values)."""
    A, W = _as_i8(pa), _as_i8(pw)
    acc = np.empty(m * n, np.int32)
    N.call("tvq_gemm_i8_acc", B.ptr(A), B.ptr(W), B.ptr(acc), m, n, k)
    return acc.reshape(m, n)


def _fp8_bytes(x) -> np.ndarray:
    a = np.asarray(x)
    if a.dtype == np.uint8:
        return np.ascontiguousarray(a)
    # list[i32] holding byte - 128 (matmul.tkv:65)
    return np.ascontiguousarray((a.astype(np.int64) + 128).astype(np.uint8))


def matmul_fp8_e4m3(pa, pw, pbias, py, m: int, n: int, k: int, scale_a: float = 1.0, scales_w=None,
                    act: int = N.ACT_NONE) -> int:
    """matmul_fp8_e4m3, matmul.tkv:46-58.  pa/pw are E4M3 bytes (uint8) or the
    reference's byte-128 int32 lists.  Optional scales as in config 3."""
    bias, nb = _bias(pbias)
    if B.is_dev(pa):
        sa = _dev_scalar(scale_a, pa)
        sw = scales_w if scales_w is not None else _dev_scalar(1.0, pa)
        N.call("tvq_dev_gemm", N.GEMM_F8, B.ptr(pa), B.ptr(pw), B.ptr(bias), None, B.ptr(py), None, m, n, k,
               B.ptr(sa), B.ptr(sw), 1 if scales_w is not None else 0, act, None, None, B.stream_of(pa))
        return 0
    A, W = _fp8_bytes(pa), _fp8_bytes(pw)
    bh = B.host_f32(bias) if bias is not None else None
    sw = B.host_f32(scales_w).ravel() if scales_w is not None else None
    Y = np.empty(m * n, np.float32)
    N.call("tvq_matmul_fp8_e4m3", B.ptr(A), B.ptr(W), B.ptr(bh), nb, B.ptr(Y), m, n, k, float(scale_a), B.ptr(sw), act)
    np.asarray(py).reshape(-1)[:m * n] = Y
    return 0


def quantize_fp8_e4m3(src, dst, mode: int = N.FP8_REF) -> int:
    """quantize_fp8_e4m3, matmul.tkv:60-66.  dst uint8 receives bytes; an
    int32 dst receives the reference's byte - 128."""
    if B.size(dst) < B.size(src):
        raise ValueError("dst too small")
    s = B.host_f32(src).ravel()
    d = np.asarray(dst)
    out = np.empty(s.size, np.uint8)
    N.call("tvq_quantize_fp8_e4m3", B.ptr(s), s.size, B.ptr(out), out.size, mode)
    if d.dtype == np.uint8:
        d.reshape(-1)[:s.size] = out
    else:
        d.reshape(-1)[:s.size] = out.astype(np.int32) - 128
    return 0


def quantize_fp8_e4m3_scaled(src, rows: int, cols: int, scales, per_row: bool, mode: int = N.FP8_REF) -> np.ndarray:
    s = B.host_f32(src).ravel()
    sc = B.host_f32(scales).ravel()
    out = np.empty(rows * cols, np.uint8)
    N.call("tvq_quantize_fp8_e4m3_scaled", B.ptr(s), rows, cols, B.ptr(out), B.ptr(sc), sc.size, 1 if per_row else 0,
           mode)
    return out.reshape(rows, cols)


def dequantize_fp8_e4m3(src, dst) -> int:
    """dequantize_fp8_e4m3, matmul.tkv:68-73"""
    if B.size(dst) < B.size(src):
        raise ValueError("dst too small")
    q = _fp8_bytes(src).ravel()
    out = np.empty(q.size, np.float32)
    N.call("tvq_dequantize_fp8_e4m3", B.ptr(q), q.size, B.ptr(out), out.size)
    np.asarray(dst).reshape(-1)[:q.size] = out
    return 0


def matmul_int8_asymmetric(pa, pw, pbias, py, m: int, n: int, k: int, scale_a: float, zp_a: int, scale_w: float,
                           zp_w: int) -> int:
    """matmul_int8_asymmetric, matmul.tkv:31-44: sum (a - zp_a)(w - zp_w),
    exact, times fl64(scale_a scale_w), plus the bias.  Zero points beyond
    +-2^17 raise TvqError (TVQ_ERR_UNSUPPORTED)."""
    bias, nb = _bias(pbias)
    if B.is_dev(pa):
        sa = _dev_scalar(scale_a, pa)
        sw = _dev_scalar(scale_w, pa)
        N.call("tvq_dev_matmul_int8_asymmetric", B.ptr(pa), B.ptr(pw), B.ptr(bias), B.ptr(py), m, n, k, B.ptr(sa),
               int(zp_a), B.ptr(sw), int(zp_w), B.stream_of(pa))
        return 0
    A, W = _as_i8(pa), _as_i8(pw)
    bh = B.host_f32(bias) if bias is not None else None
    Y = np.empty(m * n, np.float32)
    N.call("tvq_matmul_int8_asymmetric", B.ptr(A), B.ptr(W), B.ptr(bh), nb, B.ptr(Y), m, n, k, float(scale_a),
           int(zp_a), float(scale_w), int(zp_w))
    np.asarray(py).reshape(-1)[:m * n] = Y
    return 0


def _f16_bits(x, count: int) -> np.ndarray:
    a = np.asarray(x)
    if a.dtype in (np.uint16, np.float16):
        return np.ascontiguousarray(a.view(np.uint16)).reshape(-1)[:count]
    # the reference's list[i32]: two entries per element, low byte first (matmul.tkv:84-87)
    b = (a.astype(np.int64).reshape(-1)[:2 * count] & 255).astype(np.uint16)
    return np.ascontiguousarray(b[0::2] | (b[1::2] << 8))


def matmul_fp16(pa, pw, pbias, py, m: int, n: int, k: int) -> int:
    """matmul_fp16, matmul.tkv:79-96: pa / pw fp16 bit patterns (uint16 or
    float16 arrays, device uint16 / float16 tensors, or the reference's byte
    lists), y = sum a w + bias on the FP16 tensor cores (tolerance in
    include/tvq.h)."""
    bias, _nb = _bias(pbias)
    if B.is_dev(pa):
        N.call("tvq_dev_matmul_fp16", B.ptr(pa), B.ptr(pw), B.ptr(bias), B.ptr(py), m, n, k, B.stream_of(pa))
        return 0
    A, W = _f16_bits(pa, m * k), _f16_bits(pw, n * k)
    bh = B.host_f32(bias) if bias is not None else None
    Y = np.empty(m * n, np.float32)
    N.call("tvq_matmul_fp16", B.ptr(A), B.ptr(W), B.ptr(bh), _nb, B.ptr(Y), m, n, k)
    np.asarray(py).reshape(-1)[:m * n] = Y
    return 0


def quantize_fp16(src, dst) -> int:
    """quantize_fp16, matmul.tkv:106-114.  A uint16 / float16 dst receives
    the fp16 patterns; an int32 dst (the reference's list) two signed bytes
    per element and must hold 2 len(src) (ValueError otherwise)."""
    s = B.host_f32(src).ravel()
    d = np.asarray(dst)
    if d.dtype in (np.uint16, np.float16):
        if d.size < s.size:
            raise ValueError("dst too small")
        out = np.empty(s.size, np.uint16)
        N.call("tvq_quantize_fp16", B.ptr(s), s.size, B.ptr(out), out.size)
        d.reshape(-1).view(np.uint16)[:s.size] = out
        return 0
    if d.size < 2 * s.size:
        raise ValueError("dst too small (need 2 bytes/elem)")
    out = np.empty(2 * s.size, np.int32)
    N.call("tvq_quantize_fp16_i32", B.ptr(s), s.size, B.ptr(out), out.size)
    d.reshape(-1)[:2 * s.size] = out
    return 0
