"""The FP8 E4M3 encoder the kernels run (tvq_e4m3.h: e4m3_encode_fast, 32-bit
integer operations) is the reference's native_fp8_e4m3_encode
(tv/quantization/types.tkv:154-191, 228-230) for every binary32 input: a
small C++ harness compares it with the step-by-step restatement in the same
header on all 2^32 bit patterns, and with the CPU oracle's encoder on every
97th pattern (44 million).  CPU only: g++ with OpenMP, a few seconds."""
import os
import shutil
import subprocess
import tempfile

import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_e4m3_fast_encoder_matches_reference_on_all_inputs():
    lib = O.build()
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "e4m3_exhaustive")
        subprocess.check_call(["g++", "-O2", "-fopenmp", "-std=c++17", "-o", exe,
                               os.path.join(HERE, "native", "e4m3_exhaustive.cpp"), "-ldl"])
        r = subprocess.run([exe, lib, "97"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 differ from the step-by-step form" in r.stdout
