"""ctypes binding of libtvq.so (the C ABI in include/tvq.h).

Loading never falls back to anything: if the library is missing the first
call raises.  ``check(rc)`` turns a non-zero status into the Python error the
reference raises for the same condition (ValueError for size errors, as
tv/quantization/engine.tkv and matmul.tkv do) or a RuntimeError otherwise.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtvq.so")

TVQ_OK = 0
TVQ_ERR_INVALID = -1
TVQ_ERR_SIZE = -2
TVQ_ERR_CUDA = -3
TVQ_ERR_TIMEOUT = -4
TVQ_ERR_UNSUPPORTED = -5
TVQ_ERR_HANDLE = -6

ACT_NONE, ACT_RELU, ACT_GELU_TANH, ACT_GELU_ERF = 0, 1, 2, 6
FP8_REF, FP8_HW = 0, 1
GEMM_I8, GEMM_F8 = 0, 1

P = C.c_void_p
i64, i32, f32 = C.c_int64, C.c_int, C.c_float

# name -> (restype, argtypes); every function declared in include/tvq.h
SIGNATURES = {
    "tvq_version": (i32, []),
    "tvq_last_error": (i32, [C.c_char_p, i64]),
    "tvq_device_count": (i32, [P]),
    "tvq_device_error": (i32, [P]),
    "tvq_selftest_wait_timeout": (i32, [i64, P]),
    "tvq_calibrate_minmax": (i32, [P, i64, i32, P, P, P, P]),
    "tvq_calibrate_minmax_batches": (i32, [P, P, i64, i32, P, P, P, P]),
    "tvq_calibrate_per_channel_minmax": (i32, [P, i64, i64, i64, P, i64]),
    "tvq_calibrate_per_channel_params": (i32, [P, i64, i64, i64, i32, P, P, P, P, i64]),
    "tvq_quantize_int8_symmetric": (i32, [P, i64, P, i64, f32]),
    "tvq_dequantize_int8_symmetric": (i32, [P, i64, P, i64, f32]),
    "tvq_quantize_int8_per_channel": (i32, [P, i64, P, i64, i64, i64, P, i64]),
    "tvq_dequantize_int8_per_channel": (i32, [P, i64, P, i64, i64, i64, P, i64]),
    "tvq_quantize_dynamic_int8_rowwise": (i32, [P, i64, P, i64, i64, i64, P, i64]),
    "tvq_matmul_int8_per_channel": (i32, [P, P, P, i64, P, i64, i64, i64, f32, P, i64, i32]),
    "tvq_matmul_int8_symmetric": (i32, [P, P, P, i64, P, i64, i64, i64, f32, f32, i32]),
    "tvq_gemm_i8_acc": (i32, [P, P, P, i64, i64, i64]),
    "tvq_quantize_fp8_e4m3": (i32, [P, i64, P, i64, i32]),
    "tvq_quantize_fp8_e4m3_scaled": (i32, [P, i64, i64, P, P, i64, i32, i32]),
    "tvq_dequantize_fp8_e4m3": (i32, [P, i64, P, i64]),
    "tvq_matmul_fp8_e4m3": (i32, [P, P, P, i64, P, i64, i64, i64, f32, P, i32]),
    "tvq_quantize_int8_symmetric_i32": (i32, [P, i64, P, i64, f32]),
    "tvq_matmul_int8_per_channel_i32": (i32, [P, P, P, i64, P, i64, i64, i64, f32, P, i64]),
    "tvq_quantize_fp8_e4m3_i32": (i32, [P, i64, P, i64]),
    "tvq_matmul_fp8_e4m3_i32": (i32, [P, P, P, i64, P, i64, i64, i64]),
    "tvq_matmul_int8_asymmetric": (i32, [P, P, P, i64, P, i64, i64, i64, f32, i64, f32, i64]),
    "tvq_matmul_int8_asymmetric_i32": (i32, [P, P, P, i64, P, i64, i64, i64, f32, i64, f32, i64]),
    "tvq_matmul_fp16": (i32, [P, P, P, i64, P, i64, i64, i64]),
    "tvq_matmul_fp16_i32": (i32, [P, P, P, i64, P, i64, i64, i64]),
    "tvq_quantize_fp16": (i32, [P, i64, P, i64]),
    "tvq_quantize_fp16_i32": (i32, [P, i64, P, i64]),
    "tvq_dev_quantize_fp16": (i32, [P, P, i64, P]),
    "tvq_dev_matmul_fp16": (i32, [P, P, P, P, i64, i64, i64, P]),
    "tvq_dev_matmul_int8_asymmetric": (i32, [P, P, P, P, i64, i64, i64, P, i64, P, i64, P]),
    "tvq_dev_minmax_reset": (i32, [P, P]),
    "tvq_dev_minmax_accumulate": (i32, [P, i64, P, P, P]),
    "tvq_dev_minmax_finalize": (i32, [P, P, i32, P, P]),
    "tvq_dev_quantize_int8": (i32, [P, P, i64, P, P]),
    "tvq_dev_calibrate_quantize_per_channel": (i32, [P, P, P, i64, i64, P]),
    "tvq_dev_quantize_int8_per_channel": (i32, [P, P, P, i64, i64, P]),
    "tvq_dev_quantize_dynamic_rowwise": (i32, [P, P, P, i64, i64, P]),
    "tvq_dev_quantize_fp8": (i32, [P, P, i64, i64, P, i32, i32, P]),
    "tvq_dev_dequantize_fp8": (i32, [P, P, i64, P]),
    "tvq_dev_gemm": (i32, [i32, P, P, P, P, P, P, i64, i64, i64, P, P, i32, i32, P, P, P]),
    "tvq_dev_gemm_f32x3": (i32, [P, P, P, P, P, i64, i64, i64, P]),
    "tvq_dev_split_tf32": (i32, [P, P, P, i64, P]),
    "tvq_dev_gemm_f16x3": (i32, [P, P, P, P, P, P, P, i64, i64, i64, P]),
    "tvq_dev_split_f16_rows": (i32, [P, P, P, P, i64, i64, P]),
    "tvq_dev_layernorm": (i32, [P, P, P, P, P, P, P, i64, i64, C.c_double, P]),
    "tvq_dev_attention": (i32, [P, P, i64, i64, i64, P, i64, P, P, P, P, P]),
    "tvq_dev_attention_noalloc": (i32, [P, P, i64, i64, i64, P, P, P, P, P]),
    "tvq_session_create": (i32, [i32, i64, i64, i64, i64, i64, i64, C.c_double, i64, P]),
    "tvq_session_destroy": (i32, [i64]),
    "tvq_session_set_embeddings": (i32, [i64, P, P]),
    "tvq_session_set_layernorm": (i32, [i64, i64, i64, P, P]),
    "tvq_session_set_linear_f32": (i32, [i64, i64, i64, P, P, i32]),
    "tvq_session_set_linear_i8": (i32, [i64, i64, i64, P, P, P]),
    "tvq_session_get_linear_i8": (i32, [i64, i64, i64, P, P]),
    "tvq_session_set_act_scales": (i32, [i64, P, i64]),
    "tvq_session_get_act_scales": (i32, [i64, P, i64]),
    "tvq_session_prepare": (i32, [i64, P, i64, i32]),
    "tvq_session_calibrate": (i32, [i64, P, i32, i32]),
    "tvq_session_forward": (i32, [i64, P, i32, P, i64, i32, P]),
    "tvq_session_forward_async": (i32, [i64, P, i32, P, i64, P]),
    "tvq_session_join": (i32, [i64, P]),
    "tvq_session_wait": (i32, [i64, P]),
    "tvq_session_logits": (i32, [i64, P, P, P]),
    "tvq_session_run_layers": (i32, [i64, P, i32, P, i32, i32, P]),
    "tvq_dev_quantize_int4_grouped": (i32, [P, i64, i64, i64, P, P, P, P]),
    "tvq_dev_dequantize_int4_grouped": (i32, [P, P, i64, i64, i64, P, P, P]),
    "tvq_dev_permute_cols": (i32, [P, P, i64, i64, P, i32, P]),
    "tvq_dev_matmul_int4_grouped": (i32, [P, P, P, P, i64, i64, i64, i64, P, P, P]),
    "tvq_quantize_int4_grouped": (i32, [P, i64, i64, i64, P, P, P]),
    "tvq_dequantize_int4_grouped": (i32, [P, P, i64, i64, i64, P, i64, P]),
    "tvq_permute_cols": (i32, [P, P, i64, i64, P, i64, i32]),
    "tvq_matmul_int4_grouped": (i32, [P, P, P, i64, P, i64, i64, i64, i64, P, i64, P]),
    "tvq_session_hidden": (i32, [i64, P]),
    "tvq_quantize_linear": (i32, [P, P, i64, i64, i64, P, i64, i64]),
    "tvq_dequantize_linear": (i32, [P, P, i64, i64, i64, P, i64, i64]),
    "tvq_matmul_integer": (i32, [P, P, P, i64, i64, i64]),
    "tvq_qlinear_matmul": (i32, [P, f32, i64, P, f32, i64, f32, i64, P, i64, i64, i64]),
    "tvq_dynamic_quantize_linear": (i32, [P, i64, P, P, P]),
    "tvq_dev_quantize_linear": (i32, [P, P, i64, i64, i64, P, i64, i64, P]),
    "tvq_dev_dequantize_linear": (i32, [P, P, i64, i64, i64, P, i64, i64, P]),
    "tvq_dev_matmul_integer": (i32, [P, P, P, i64, i64, i64, P]),
    "tvq_dev_qlinear_matmul": (i32, [P, f32, i64, P, f32, i64, f32, i64, P, i64, i64, i64, P]),
    "tvq_dev_dynamic_quantize_linear": (i32, [P, i64, P, P, P, P]),
    "tvq_calibrate_kl": (i32, [P, i64, i64, i64, P, P, P, P]),
    "tvq_calibrate_percentile": (i32, [P, i64, f32, i32, P, P, P, P]),
    "tvq_calibrate_mse": (i32, [P, i64, i64, P, P, P, P]),
    "tvq_dev_calibrate_mse_curve": (i32, [P, i64, i64, P, P, P, P]),
    "tvq_session_launches": (i32, [i64, P]),
    "tvq_session_sync": (i32, [i64]),
    "tvq_session_set_profiling": (i32, [i64, i32]),
    "tvq_session_stage_times": (i32, [i64, P, i64]),
}

_lib = None
_lock = threading.Lock()


class TvqError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def lib():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    "libtvq.so is not built (%s); run tokenvector/inference_b200/build.py -- "
                    "there is no CPU fallback" % LIB_PATH)
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().tvq_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(rc: int) -> None:
    if rc == TVQ_OK:
        return
    msg = last_error()
    if rc == TVQ_ERR_SIZE:
        raise ValueError(msg)
    raise TvqError(rc, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
