"""CPU oracle for the PTQ linear path -- TEST INFRASTRUCTURE ONLY.

ctypes bindings over ``liboracle.so`` (built from ``tvq_oracle.c`` by the
Makefile beside it).  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` may import this package, and only as the
checker: the product path in ``tokenvector.inference_b200`` never calls it.

Each wrapper names the reference function it restates (tv/... path:line,
relative to the TokenVector.Inference repository root).  Parity pins: see the
header of tvq_oracle.c -- the INT8 GEMM and the f64 epilogue model have no
reference fixture (parity unpinned beyond the restatement); calibrate_minmax,
the quantize round trip and the FP8 round trip are pinned by the reference's
own tests.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


class QParams(C.Structure):
    """QuantParams, tv/quantization/types.tkv:17-27."""

    _fields_ = [("scale", C.c_float), ("zero_point", C.c_int64),
                ("min_val", C.c_float), ("max_val", C.c_float)]


def build(force: bool = False) -> str:
    if force or not os.path.exists(_LIB_PATH) or \
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "tvq_oracle.c")):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        i64, f32, f64, i32 = C.c_int64, C.c_float, C.c_double, C.c_int
        sig = {
            "tvo_f64_to_f32_bits": (C.c_uint32, [f64]),
            "tvo_f32_bits_to_f64": (f64, [C.c_uint32]),
            "tvo_rne_rshift": (i64, [i64, i64]),
            "tvo_fp8_encode": (i32, [f32, i32, i32, i32, i32, i32]),
            "tvo_fp8_decode": (f32, [i32, i32, i32, i32, i32]),
            "tvo_e4m3_encode": (i32, [f32]),
            "tvo_e4m3_decode": (f32, [i32]),
            "tvo_e5m2_encode": (i32, [f32]),
            "tvo_e5m2_decode": (f32, [i32]),
            "tvo_f16_encode": (i32, [f32]),
            "tvo_f16_decode": (f32, [i32]),
            "tvo_calibrate_minmax": (QParams, [P, i64, i32]),
            "tvo_calibrate_per_channel_minmax": (i32, [P, i64, i64, i64, i32, P]),
            "tvo_quantize_int8_symmetric": (i32, [P, i64, P, i64, f32]),
            "tvo_dequantize_int8_symmetric": (i32, [P, i64, P, i64, f32]),
            "tvo_quantize_int8_per_channel": (i32, [P, i64, P, i64, i64, i64, P, i64]),
            "tvo_dequantize_int8_per_channel": (i32, [P, i64, P, i64, i64, i64, P, i64]),
            "tvo_quantize_dynamic_int8_rowwise": (i32, [P, i64, P, i64, i64, i64, P, i64]),
            "tvo_dot_int8": (i64, [P, P, i64]),
            "tvo_gemm_i8_acc_i32": (i32, [P, P, P, i64, i64, i64]),
            "tvo_matmul_int8_per_channel": (i32, [P, P, P, i64, P, i64, i64, i64, f32, P, i64]),
            "tvo_matmul_int8_symmetric": (i32, [P, P, P, i64, P, i64, i64, i64, f32, f32]),
            "tvo_matmul_int8_asymmetric": (i32, [P, P, P, i64, P, i64, i64, i64, f32, i64, f32, i64]),
            "tvo_quantize_fp16": (i32, [P, i64, P]),
            "tvo_matmul_fp16": (i32, [P, P, P, i64, P, i64, i64, i64]),
            "tvo_quantize_fp8_e4m3": (i32, [P, i64, P]),
            "tvo_quantize_fp8_e4m3_scaled": (i32, [P, i64, i64, P, P, i32]),
            "tvo_dequantize_fp8_e4m3": (i32, [P, i64, P]),
            "tvo_matmul_fp8_e4m3": (i32, [P, P, P, i64, P, i64, i64, i64, f32, P]),
            "tvo_gelu_tanh": (f32, [f32]),
            "tvo_erf_as": (f32, [f32]),
            "tvo_gelu_erf": (f32, [f32]),
            "tvo_gelu_erf_inplace": (None, [P, i64]),
            "tvo_layernorm": (None, [P, P, P, P, i64, i64, f64]),
            "tvo_embed": (None, [P, P, P, P, P, i64, i64]),
            "tvo_attention_causal": (None, [P, P, i64, i64, i64, P, i64]),
            "tvo_add": (None, [P, P, P, i64]),
            "tvo_lm_head": (None, [P, P, P, i64, i64, i64]),
            "tvo_lm_head_plain": (None, [P, P, P, i64, i64, i64]),
            "tvo_matmul_int8_per_channel_scalar": (i32, [P, P, P, i64, P, i64, i64, i64, f32, P, i64]),
            "tvo_gi_noise": (None, [P, i64, i64, f64]),
            "tvo_quantize_linear": (i32, [P, P, i64, i64, i64, P, i64, i64]),
            "tvo_dequantize_linear": (i32, [P, P, i64, i64, i64, P, i64, i64]),
            "tvo_matmul_integer": (i32, [P, P, P, i64, i64, i64]),
            "tvo_qlinear_matmul": (i32, [P, f32, i64, P, f32, i64, f32, i64, P, i64, i64, i64]),
            "tvo_dynamic_quantize_linear": (i32, [P, i64, P, P, P]),
            "tvo_calibrate_kl": (QParams, [P, i64, i64, i64]),
            "tvo_calibrate_percentile": (QParams, [P, i64, f32, i32, P]),
            "tvo_calibrate_mse": (QParams, [P, i64, i64]),
            "tvo_calibrate_mse_curve": (None, [P, i64, i64, P]),
            "tvo_quantize_int4_grouped": (i32, [P, i64, i64, i64, P, P]),
            "tvo_dequantize_int4_grouped": (i32, [P, P, i64, i64, i64, P]),
            "tvo_quantize_int4_grouped_asym": (i32, [P, i64, i64, i64, P, P, P]),
            "tvo_dequantize_int4_grouped_asym": (i32, [P, P, i64, i64, i64, P, P]),
            "tvo_permute_cols": (i32, [P, P, i64, i64, P, i32]),
            "tvo_matmul_int4_grouped": (i32, [P, P, P, i64, P, i64, i64, i64, i64, P, P]),
            "tvo_num_threads": (i32, []),
            "tvo_set_num_threads": (None, [i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be contiguous"
    return a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i8(a):
    return np.ascontiguousarray(a, dtype=np.int8)


# ---------------------------------------------------------------- codecs
def f64_to_f32_bits(x: float) -> int:
    """tv/runtime/f32_bits.tkv:6-57"""
    return int(lib().tvo_f64_to_f32_bits(float(x)))


def f32_bits_to_f64(b: int) -> float:
    """tv/runtime/f32_bits.tkv:60-74"""
    return float(lib().tvo_f32_bits_to_f64(int(b) & 0xFFFFFFFF))


def rne_rshift(v: int, s: int) -> int:
    """_qt_rne_rshift, tv/quantization/types.tkv:71-93"""
    return int(lib().tvo_rne_rshift(v, s))


def e4m3_encode(x: float) -> int:
    """native_fp8_e4m3_encode, tv/quantization/types.tkv:228-230 (byte)"""
    return int(lib().tvo_e4m3_encode(float(x)))


def e4m3_decode(v: int) -> float:
    """native_fp8_e4m3_decode, tv/quantization/types.tkv:232-233"""
    return float(lib().tvo_e4m3_decode(int(v)))


def e5m2_encode(x: float) -> int:
    return int(lib().tvo_e5m2_encode(float(x)))


def e5m2_decode(v: int) -> float:
    return float(lib().tvo_e5m2_decode(int(v)))


def f16_encode(x: float) -> int:
    return int(lib().tvo_f16_encode(float(x)))


def f16_decode(v: int) -> float:
    return float(lib().tvo_f16_decode(int(v)))


def quantize_fp8_e4m3(src) -> np.ndarray:
    """quantize_fp8_e4m3, tv/quantization/matmul.tkv:60-66 (byte form)."""
    s = _f32(src)
    out = np.empty(s.shape, dtype=np.uint8)
    lib().tvo_quantize_fp8_e4m3(_p(s), s.size, _p(out))
    return out


def quantize_fp8_e4m3_scaled(src, scales, per_row: bool) -> np.ndarray:
    s = _f32(src)
    rows = s.shape[0] if s.ndim == 2 else 1
    cols = s.size // rows
    sc = _f32(np.atleast_1d(scales))
    out = np.empty(s.shape, dtype=np.uint8)
    lib().tvo_quantize_fp8_e4m3_scaled(_p(s), rows, cols, _p(out), _p(sc), 1 if per_row else 0)
    return out


def dequantize_fp8_e4m3(src) -> np.ndarray:
    s = np.ascontiguousarray(src, dtype=np.uint8)
    out = np.empty(s.shape, dtype=np.float32)
    lib().tvo_dequantize_fp8_e4m3(_p(s), s.size, _p(out))
    return out


# ---------------------------------------------------------------- engine.tkv
def calibrate_minmax(data, symmetric: int = 1) -> QParams:
    """calibrate_minmax, tv/quantization/engine.tkv:13-36"""
    d = _f32(data).ravel()
    return lib().tvo_calibrate_minmax(_p(d), d.size, int(symmetric))


def calibrate_per_channel_minmax(data, rows: int, cols: int, symmetric: int = 1):
    """calibrate_per_channel_minmax, tv/quantization/engine.tkv:202-213"""
    d = _f32(data).ravel()
    out = (QParams * max(rows, 1))()
    rc = lib().tvo_calibrate_per_channel_minmax(_p(d), d.size, rows, cols, int(symmetric), C.cast(out, C.c_void_p))
    if rc != 0:
        raise ValueError("rows/cols must be > 0 and data >= rows*cols")
    return [out[i] for i in range(rows)]


def per_channel_scales(w, rows: int, cols: int) -> np.ndarray:
    return np.array([q.scale for q in calibrate_per_channel_minmax(w, rows, cols, 1)], dtype=np.float32)


def quantize_int8_symmetric(src, scale: float) -> np.ndarray:
    """quantize_int8_symmetric, tv/quantization/engine.tkv:216-226"""
    s = _f32(src)
    out = np.empty(s.shape, dtype=np.int8)
    lib().tvo_quantize_int8_symmetric(_p(s), s.size, _p(out), out.size, float(scale))
    return out


def dequantize_int8_symmetric(src, scale: float) -> np.ndarray:
    """dequantize_int8_symmetric, tv/quantization/engine.tkv:229-234"""
    s = _i8(src)
    out = np.empty(s.shape, dtype=np.float32)
    lib().tvo_dequantize_int8_symmetric(_p(s), s.size, _p(out), out.size, float(scale))
    return out


def quantize_int8_per_channel(src, rows: int, cols: int, scales) -> np.ndarray:
    """quantize_int8_per_channel, tv/quantization/engine.tkv:237-250"""
    s = _f32(src)
    sc = _f32(scales)
    out = np.empty(s.shape, dtype=np.int8)
    rc = lib().tvo_quantize_int8_per_channel(_p(s), s.size, _p(out), out.size, rows, cols, _p(sc), sc.size)
    if rc != 0:
        raise ValueError("span too small")
    return out


def dequantize_int8_per_channel(src, rows: int, cols: int, scales) -> np.ndarray:
    s = _i8(src)
    sc = _f32(scales)
    out = np.empty(s.shape, dtype=np.float32)
    rc = lib().tvo_dequantize_int8_per_channel(_p(s), s.size, _p(out), out.size, rows, cols, _p(sc), sc.size)
    if rc != 0:
        raise ValueError("span too small")
    return out


def quantize_dynamic_int8_rowwise(src, rows: int, cols: int):
    """quantize_dynamic_int8_rowwise, tv/quantization/engine.tkv:266-285"""
    s = _f32(src)
    out = np.empty(s.shape, dtype=np.int8)
    sc = np.empty(rows, dtype=np.float32)
    rc = lib().tvo_quantize_dynamic_int8_rowwise(_p(s), s.size, _p(out), out.size, rows, cols, _p(sc), sc.size)
    if rc != 0:
        raise ValueError("span too small")
    return out, sc


# ---------------------------------------------------------------- matmul.tkv
def dot_int8(a, b) -> int:
    a = _i8(a)
    b = _i8(b)
    return int(lib().tvo_dot_int8(_p(a), _p(b), a.size))


def gemm_i8_acc(A, W) -> np.ndarray:
    """int32 accumulators of _dot_int8 over every (m, n)."""
    A = _i8(A)
    W = _i8(W)
    m, k = A.shape
    n = W.shape[0]
    out = np.empty((m, n), dtype=np.int32)
    lib().tvo_gemm_i8_acc_i32(_p(A), _p(W), _p(out), m, n, k)
    return out


def matmul_int8_per_channel_scalar(A, W, bias, scale_a: float, scales_w) -> np.ndarray:
    """The faithful single-thread scalar form of matmul_int8_per_channel
    (matmul.tkv:17-29, _dot_int8 :116-127): the one-core CPU baseline."""
    A = _i8(A)
    W = _i8(W)
    m, k = A.shape
    n = W.shape[0]
    b = _f32(bias) if bias is not None else np.zeros(0, np.float32)
    sw = _f32(scales_w)
    Y = np.empty((m, n), dtype=np.float32)
    rc = lib().tvo_matmul_int8_per_channel_scalar(_p(A), _p(W), _p(b) if b.size else None, b.size, _p(Y), m, n, k,
                                                  float(scale_a), _p(sw), sw.size)
    if rc != 0:
        raise ValueError("scales_w smaller than N")
    return Y


def matmul_int8_per_channel(A, W, bias, scale_a: float, scales_w) -> np.ndarray:
    """matmul_int8_per_channel, tv/quantization/matmul.tkv:17-29"""
    A = _i8(A)
    W = _i8(W)
    m, k = A.shape
    n = W.shape[0]
    b = _f32(bias) if bias is not None else np.zeros(0, np.float32)
    sw = _f32(scales_w)
    Y = np.empty((m, n), dtype=np.float32)
    rc = lib().tvo_matmul_int8_per_channel(_p(A), _p(W), _p(b) if b.size else None, b.size, _p(Y), m, n, k,
                                           float(scale_a), _p(sw), sw.size)
    if rc != 0:
        raise ValueError("scales_w smaller than N")
    return Y


def matmul_int8_symmetric(A, W, bias, scale_a: float, scale_w: float) -> np.ndarray:
    """matmul_int8_symmetric, tv/quantization/matmul.tkv:4-15"""
    A = _i8(A)
    W = _i8(W)
    m, k = A.shape
    n = W.shape[0]
    b = _f32(bias) if bias is not None else np.zeros(0, np.float32)
    Y = np.empty((m, n), dtype=np.float32)
    lib().tvo_matmul_int8_symmetric(_p(A), _p(W), _p(b) if b.size else None, b.size, _p(Y), m, n, k,
                                    float(scale_a), float(scale_w))
    return Y


def matmul_int8_asymmetric(A, W, bias, scale_a, zp_a, scale_w, zp_w) -> np.ndarray:
    """matmul_int8_asymmetric, tv/quantization/matmul.tkv:31-44"""
    A = _i8(A)
    W = _i8(W)
    m, k = A.shape
    n = W.shape[0]
    b = _f32(bias) if bias is not None else np.zeros(0, np.float32)
    Y = np.empty((m, n), dtype=np.float32)
    lib().tvo_matmul_int8_asymmetric(_p(A), _p(W), _p(b) if b.size else None, b.size, _p(Y), m, n, k,
                                     float(scale_a), int(zp_a), float(scale_w), int(zp_w))
    return Y


def quantize_fp16(src) -> np.ndarray:
    """quantize_fp16, tv/quantization/matmul.tkv:106-114 (uint16 patterns)."""
    s = _f32(src)
    out = np.empty(s.shape, dtype=np.uint16)
    lib().tvo_quantize_fp16(_p(s), s.size, _p(out))
    return out


def matmul_fp16(A, W, bias) -> np.ndarray:
    """matmul_fp16, tv/quantization/matmul.tkv:79-96 (uint16 fp16 operands)."""
    A = np.ascontiguousarray(A, dtype=np.uint16)
    W = np.ascontiguousarray(W, dtype=np.uint16)
    m, k = A.shape
    n = W.shape[0]
    b = _f32(bias) if bias is not None else np.zeros(0, np.float32)
    Y = np.empty((m, n), dtype=np.float32)
    lib().tvo_matmul_fp16(_p(A), _p(W), _p(b) if b.size else None, b.size, _p(Y), m, n, k)
    return Y


def matmul_fp8_e4m3(A, W, bias, scale_a: float = 1.0, scales_w=None) -> np.ndarray:
    """matmul_fp8_e4m3, tv/quantization/matmul.tkv:46-58 (byte operands)."""
    A = np.ascontiguousarray(A, dtype=np.uint8)
    W = np.ascontiguousarray(W, dtype=np.uint8)
    m, k = A.shape
    n = W.shape[0]
    b = _f32(bias) if bias is not None else np.zeros(0, np.float32)
    sw = _f32(scales_w) if scales_w is not None else None
    Y = np.empty((m, n), dtype=np.float32)
    lib().tvo_matmul_fp8_e4m3(_p(A), _p(W), _p(b) if b.size else None, b.size, _p(Y), m, n, k,
                              float(scale_a), _p(sw))
    return Y


# ---------------------------------------------------------------- activations / GPT-2 glue
def gelu_tanh(x: float) -> float:
    return float(lib().tvo_gelu_tanh(float(x)))


def erf_as(x: float) -> float:
    return float(lib().tvo_erf_as(float(x)))


def gelu_erf(x: float) -> float:
    return float(lib().tvo_gelu_erf(float(x)))


def gelu_erf_array(x) -> np.ndarray:
    a = _f32(x).copy()
    lib().tvo_gelu_erf_inplace(_p(a), a.size)
    return a


def layernorm(x, g, b, eps: float = 1e-6) -> np.ndarray:
    x = _f32(x)
    n, h = x.shape
    out = np.empty_like(x)
    lib().tvo_layernorm(_p(x), _p(_f32(g)), _p(_f32(b)), _p(out), n, h, float(eps))
    return out


def embed(ids, pos, wte, wpe) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    pos = np.ascontiguousarray(pos, dtype=np.int64)
    wte = _f32(wte)
    wpe = _f32(wpe)
    h = wte.shape[1]
    if pos.size != ids.size or wpe.shape[1] != h:
        raise ValueError("embed: one position per token and equal widths are required")
    if ids.size and (ids.min() < 0 or ids.max() >= wte.shape[0] or pos.min() < 0 or pos.max() >= wpe.shape[0]):
        raise ValueError("embed: token id or position out of range")
    out = np.empty((ids.size, h), dtype=np.float32)
    lib().tvo_embed(_p(ids), _p(pos), _p(wte), _p(wpe), _p(out), ids.size, h)
    return out


def attention_causal(qkv, nheads: int, seg) -> np.ndarray:
    qkv = _f32(qkv)
    n = qkv.shape[0]
    h = qkv.shape[1] // 3
    seg = np.ascontiguousarray(seg, dtype=np.int64)
    ctx = np.zeros((n, h), dtype=np.float32)
    lib().tvo_attention_causal(_p(qkv), _p(ctx), n, h, nheads, _p(seg), seg.size - 1)
    return ctx


def add(a, b) -> np.ndarray:
    a = _f32(a)
    b = _f32(b)
    out = np.empty_like(a)
    lib().tvo_add(_p(a), _p(b), _p(out), a.size)
    return out


def lm_head(x, wte, plain: bool = False) -> np.ndarray:
    """Tied LM head, gpt2_ref.tkv:603-610 (f64 sums in k order); plain=True
    runs the one-output-at-a-time loop (same bits, slower)."""
    x = _f32(x)
    wte = _f32(wte)
    n, h = x.shape
    vocab = wte.shape[0]
    out = np.empty((n, vocab), dtype=np.float32)
    (lib().tvo_lm_head_plain if plain else lib().tvo_lm_head)(_p(x), _p(wte), _p(out), n, vocab, h)
    return out


def gi_noise(n: int, seed: int, mult: float = 0.02) -> np.ndarray:
    """_gi_noise, tv/training/gpt2_ref.tkv:1977-1991"""
    out = np.empty(n, dtype=np.float32)
    lib().tvo_gi_noise(_p(out), n, seed, float(mult))
    return out


def num_threads() -> int:
    return int(lib().tvo_num_threads())


def set_num_threads(n: int) -> None:
    lib().tvo_set_num_threads(int(n))


# ---------------------------------------------------------------- ONNX QDQ operators (session.tkv)
def _axis_split(shape, axis: int, nsc: int):
    """(outer, dim, inner) of `shape` at `axis` (negative counts from the end,
    session.tkv:1926-1940); per tensor when nsc == 1."""
    shape = list(shape)
    if nsc == 1:
        n = int(np.prod(shape)) if shape else 1
        return 1, n, 1
    ax = axis if axis >= 0 else axis + len(shape)
    outer = int(np.prod(shape[:ax])) if ax > 0 else 1
    inner = int(np.prod(shape[ax + 1:])) if ax + 1 < len(shape) else 1
    return outer, int(shape[ax]), inner


def quantize_linear(x, scales, zero_point: int = 0, axis: int = 1) -> np.ndarray:
    """_exec_quantize_linear, tv/runtime/session.tkv:1896-1953"""
    x = _f32(x)
    sc = _f32(np.atleast_1d(scales))
    outer, dim, inner = _axis_split(x.shape, axis, sc.size)
    y = np.empty(x.shape, np.int8)
    if lib().tvo_quantize_linear(_p(x), _p(y), outer, dim, inner, _p(sc), sc.size, int(zero_point)) != 0:
        raise ValueError("one scale, or one per channel of the axis")
    return y


def dequantize_linear(x, scales, zero_point: int = 0, axis: int = 1) -> np.ndarray:
    """_exec_dequantize_linear, tv/runtime/session.tkv:1955-1990"""
    x = _i8(x)
    sc = _f32(np.atleast_1d(scales))
    outer, dim, inner = _axis_split(x.shape, axis, sc.size)
    y = np.empty(x.shape, np.float32)
    if lib().tvo_dequantize_linear(_p(x), _p(y), outer, dim, inner, _p(sc), sc.size, int(zero_point)) != 0:
        raise ValueError("one scale, or one per channel of the axis")
    return y


def matmul_integer(a, b) -> np.ndarray:
    """_exec_matmul_integer, tv/runtime/session.tkv:2789-2851 (B is [K, N])"""
    a = _i8(a)
    b = _i8(b)
    m, k = a.shape
    n = b.shape[1]
    y = np.empty((m, n), np.int32)
    lib().tvo_matmul_integer(_p(a), _p(b), _p(y), m, k, n)
    return y


def qlinear_matmul(a, sa, zpa, b, sw, zpw, sy, zpy) -> np.ndarray:
    """_exec_qlinear_matmul, tv/runtime/session.tkv:1992-2071 (B is [K, N])"""
    a = _i8(a)
    b = _i8(b)
    m, k = a.shape
    n = b.shape[1]
    y = np.empty((m, n), np.int8)
    lib().tvo_qlinear_matmul(_p(a), float(sa), int(zpa), _p(b), float(sw), int(zpw), float(sy), int(zpy), _p(y),
                             m, k, n)
    return y


def dynamic_quantize_linear(x):
    """_exec_dyn_quant, tv/runtime/session.tkv:2853-2905 -> (int8 y, scale, zero point)"""
    x = _f32(x).ravel()
    y = np.empty(x.size, np.int8)
    s = np.zeros(1, np.float32)
    z = np.zeros(1, np.float32)
    if lib().tvo_dynamic_quantize_linear(_p(x), x.size, _p(y), _p(s), _p(z)) != 0:
        raise ValueError("empty input")
    return y, float(s[0]), float(z[0])


# ---------------------------------------------------------------- calibration methods (engine.tkv:42-197)
def calibrate_kl(data, num_bins: int = 2048, target_bins: int = 128) -> QParams:
    """calibrate_kl, tv/quantization/engine.tkv:42-122"""
    d = _f32(data).ravel()
    return lib().tvo_calibrate_kl(_p(d), d.size, int(num_bins), int(target_bins))


def calibrate_percentile(data, percentile: float = 99.99, symmetric: int = 1) -> QParams:
    """calibrate_percentile, tv/quantization/engine.tkv:125-162"""
    d = _f32(data).ravel()
    err = C.c_int(0)
    r = lib().tvo_calibrate_percentile(_p(d), d.size, float(percentile), int(symmetric), C.byref(err))
    if err.value:
        raise ValueError("percentile must be in (0, 100]")
    return r


def calibrate_mse(data, num_candidates: int = 50) -> QParams:
    """calibrate_mse, tv/quantization/engine.tkv:165-197"""
    d = _f32(data).ravel()
    return lib().tvo_calibrate_mse(_p(d), d.size, int(num_candidates))


def calibrate_mse_curve(data, num_candidates: int = 50) -> np.ndarray:
    d = _f32(data).ravel()
    out = np.empty(num_candidates, np.float64)
    lib().tvo_calibrate_mse_curve(_p(d), d.size, int(num_candidates), _p(out))
    return out



# ---------------------------------------------------------------- tv/quantization/int4.tkv
def _i4_check(rc):
    if rc != 0:
        raise ValueError("cols must be an even multiple of group_size (or a permutation index is out of range)")


def quantize_int4_grouped(src, rows: int, cols: int, group_size: int):
    """int4.tkv:27-48 -> (packed uint8 [rows, cols/2], scales f32 [rows, cols/group_size])."""
    x = _f32(src).reshape(rows, cols)
    packed = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows, max(cols // max(group_size, 1), 1)), np.float32)
    _i4_check(lib().tvo_quantize_int4_grouped(_p(x), rows, cols, group_size, _p(packed), _p(scales)))
    return packed, scales


def dequantize_int4_grouped(packed, rows: int, cols: int, group_size: int, scales) -> np.ndarray:
    """int4.tkv:51-64."""
    pk = np.ascontiguousarray(packed, np.uint8)
    sc = _f32(scales)
    out = np.empty((rows, cols), np.float32)
    _i4_check(lib().tvo_dequantize_int4_grouped(_p(pk), _p(out), rows, cols, group_size, _p(sc)))
    return out


def quantize_int4_grouped_asym(src, rows: int, cols: int, group_size: int):
    """int4.tkv:68-150 -> (packed, scales f32, zero points int64)."""
    x = _f32(src).reshape(rows, cols)
    ng = cols // max(group_size, 1)
    packed = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows, max(ng, 1)), np.float32)
    zps = np.zeros((rows, max(ng, 1)), np.int64)
    _i4_check(lib().tvo_quantize_int4_grouped_asym(_p(x), rows, cols, group_size, _p(packed), _p(scales), _p(zps)))
    return packed, scales, zps


def dequantize_int4_grouped_asym(packed, rows: int, cols: int, group_size: int, scales, zps) -> np.ndarray:
    """int4.tkv:153-164."""
    pk = np.ascontiguousarray(packed, np.uint8)
    sc = _f32(scales)
    zp = np.ascontiguousarray(zps, np.int64)
    out = np.empty((rows, cols), np.float32)
    _i4_check(lib().tvo_dequantize_int4_grouped_asym(_p(pk), _p(out), rows, cols, group_size, _p(sc), _p(zp)))
    return out


def permute_cols(src, rows: int, cols: int, perm, inverse: bool = False) -> np.ndarray:
    """permute_cols / inv_permute_cols, int4.tkv:169-184."""
    x = _f32(src).reshape(rows, cols)
    pm = np.ascontiguousarray(perm, np.int64)
    if pm.size != cols:
        raise ValueError("perm length must equal cols")
    out = np.empty_like(x)
    _i4_check(lib().tvo_permute_cols(_p(x), _p(out), rows, cols, _p(pm), 1 if inverse else 0))
    return out


def matmul_int4_grouped(A, packed, bias, group_size: int, scales, perm=None) -> np.ndarray:
    """matmul_int4_grouped (int4.tkv:213-239); with perm the act-order form
    matmul_int4_grouped_ordered (:187-208).  A f32 [m, k], packed [n, k/2]."""
    a = _f32(A)
    m, k = a.shape
    pk = np.ascontiguousarray(packed, np.uint8)
    n = pk.shape[0]
    sc = _f32(scales)
    b = _f32(bias) if bias is not None and len(bias) else np.zeros(0, np.float32)
    pm = np.ascontiguousarray(perm, np.int64) if perm is not None else None
    y = np.empty((m, n), np.float32)
    _i4_check(lib().tvo_matmul_int4_grouped(_p(a), _p(pk), _p(b) if b.size else None, b.size, _p(y), m, n, k,
                                            group_size, _p(sc), _p(pm) if pm is not None else None))
    return y
