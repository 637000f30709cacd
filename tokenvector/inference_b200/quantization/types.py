"""Mirror of tv/quantization/types.tkv: QuantParams and the FP8-E4M3 codec.

The codec runs on the GPU (libtvq's reference encoder/decoder); the scalar
helpers here call it on one-element buffers, as the reference's scalar
functions are called per element.
"""
from __future__ import annotations

import numpy as np

from .. import _native as N
from . import _buf as B

# enum -> module constants, types.tkv:7-15
QuantPrecision_FP32 = 0
QuantPrecision_FP16 = 1
QuantPrecision_INT8_Symmetric = 2
QuantPrecision_INT8_Asymmetric = 3
QuantPrecision_FP8_E4M3 = 4
QuantPrecision_FP8_E5M2 = 5
CalibrationMethod_MinMax = 0
CalibrationMethod_KLDivergence = 1
CalibrationMethod_Percentile = 2

_F32_MAX = float(np.finfo(np.float32).max)


class QuantParams:
    """types.tkv:17-27: scale f32, zero_point i64, min_val/max_val f32."""

    __slots__ = ("scale", "zero_point", "min_val", "max_val")

    def __init__(self, scale: float = 1.0, zero_point: int = 0, min_v: float = -_F32_MAX, max_v: float = _F32_MAX):
        self.scale = float(np.float32(scale))
        self.zero_point = int(zero_point)
        self.min_val = float(np.float32(min_v))
        self.max_val = float(np.float32(max_v))

    def __repr__(self):
        return "QuantParams(scale=%r, zero_point=%r, min_val=%r, max_val=%r)" % (
            self.scale, self.zero_point, self.min_val, self.max_val)


def identity() -> QuantParams:
    """types.tkv:244-245"""
    return QuantParams(1.0, 0, -_F32_MAX, _F32_MAX)


def native_fp8_e4m3_encode(x: float) -> int:
    """types.tkv:228-230 -> byte (0..255)."""
    src = np.array([x], np.float32)
    dst = np.zeros(1, np.uint8)
    N.call("tvq_quantize_fp8_e4m3", B.ptr(src), 1, B.ptr(dst), 1, N.FP8_REF)
    return int(dst[0])


def native_fp8_e4m3_decode(v: int) -> float:
    """types.tkv:232-233"""
    src = np.array([int(v) & 0xFF], np.uint8)
    dst = np.zeros(1, np.float32)
    N.call("tvq_dequantize_fp8_e4m3", B.ptr(src), 1, B.ptr(dst), 1)
    return float(dst[0])


class FP8E4M3:
    """types.tkv:30-37"""

    __slots__ = ("value",)

    def __init__(self, v: int = 0):
        self.value = int(v) & 0xFF

    def to_float(self) -> float:
        return native_fp8_e4m3_decode(self.value)


def fp8e4m3_from_float(x: float) -> FP8E4M3:
    """types.tkv:248-249"""
    return FP8E4M3(native_fp8_e4m3_encode(x))
