"""The FP16 encoder the quantize kernel runs (tvq_f16.h: f16_encode_fast,
32-bit integer operations) is the reference's native_f16_encode
(tv/quantization/types.tkv:95-127) for every binary32 input: a small C++
harness compares it with the step-by-step restatement in the same header on
all 2^32 bit patterns, and with the CPU oracle's encoder on every 97th
pattern.  CPU only: g++ with OpenMP, a few seconds."""
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_f16_fast_encoder_matches_reference_on_all_inputs():
    lib = O.build()
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "f16_exhaustive")
        subprocess.check_call(["g++", "-O2", "-fopenmp", "-std=c++17", "-o", exe,
                               os.path.join(HERE, "native", "f16_exhaustive.cpp"), "-ldl"])
        r = subprocess.run([exe, lib, "97"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 differ from the step-by-step form" in r.stdout


def test_oracle_fp16_known_answers():
    # inference_tests.tkv:656-664: the 2x2 identity through quantize_fp16 and
    # matmul_fp16 (a zero bias of length 2) gives y[0] = y[3] = 1
    a = O.quantize_fp16(np.array([1.0, 0.0, 0.0, 1.0], np.float32)).reshape(2, 2)
    y = O.matmul_fp16(a, a, np.zeros(2, np.float32))
    assert abs(y[0, 0] - 1.0) < 0.001 and abs(y[1, 1] - 1.0) < 0.001
    assert y[0, 1] == 0.0 and y[1, 0] == 0.0
    # the encoder's departures from IEEE rounding (types.tkv:95-127)
    assert O.f16_encode(6.1e-5) == 0x03FF        # rounds up out of the subnormals: stays 0x3FF
    assert O.f16_encode(float("nan")) == 0x7E00  # one quiet NaN, sign dropped
    assert O.f16_encode(65520.0) == 0x7C00       # above the largest finite: Inf
    assert O.f16_encode(-0.0) == 0
    # FP16.to_float reads exponent 31 as +-Inf, NaN patterns included (f32_bits_to_f64)
    assert O.f16_decode(0x7E00) == float("inf") and O.f16_decode(0xFC01) == float("-inf")
