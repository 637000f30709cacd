"""Pin the CPU oracle against the reference's own tests and fixtures.

Known-answer tests come from tv/tests/gap_tests.tkv:159-240 and
tv/tests/inference_tests.tkv:634-665, 895-921 of TokenVector.Inference; the
GPT-2 glue is checked against the torch fixtures tv/tests/fixtures/g2_*.txt
(converted to tests/golden/g2_reduced.npz by tests/golden/make_golden.py).
Hand-derived cases cover the edges the reference does not test: ties at .5,
the 1e-8 floors, E4M3 saturation and subnormal carry.
"""
import math
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "g2_reduced.npz")


def test_calibrate_minmax_known_answer():
    # gap_tests.tkv:159-168
    p = O.calibrate_minmax(np.array([-12.7, 0.0, 6.35, 12.7], np.float32), 1)
    assert abs(p.scale - 0.1) < 1e-5
    assert p.zero_point == 0


def test_quantize_roundtrip_known_answer():
    # gap_tests.tkv:171-193: max |x - dq| <= scale + 1e-6
    x = np.array([-1.5, -0.5, 0.0, 0.5, 1.5], np.float32)
    p = O.calibrate_minmax(x, 1)
    q = O.quantize_int8_symmetric(x, p.scale)
    dq = O.dequantize_int8_symmetric(q, p.scale)
    assert np.abs(x - dq).max() <= p.scale + 1e-6
    assert q.tolist() == [-127, -42, 0, 42, 127]


def test_fp8_roundtrip_known_answer():
    # gap_tests.tkv:196-240
    for v in [0.0, 0.5, 1.0, -1.0, 2.5, 16.0]:
        rec = O.e4m3_decode(O.e4m3_encode(v))
        assert abs(v - rec) / (abs(v) + 1e-5) < 0.15
    for v in [0.0, 0.25, 1.0, -2.0, 64.0, 512.0]:
        rec = O.e5m2_decode(O.e5m2_encode(v))
        assert abs(v - rec) / (abs(v) + 1e-5) < 0.25


def test_fp16_identity_known_answer():
    # inference_tests.tkv:656-664: FP16 of 1.0 is 0x3C00 and decodes back
    assert O.f16_encode(1.0) == 0x3C00
    assert O.f16_decode(0x3C00) == 1.0


def test_matmul_integer_known_answer():
    # inference_tests.tkv:895-921: A=[[1,2],[3,4]], B=ones[K,N] -> [3,3,7,7]
    A = np.array([[1, 2], [3, 4]], np.int8)
    W = np.ones((2, 2), np.int8)           # B^T in the [N,K] layout
    assert O.gemm_i8_acc(A, W).ravel().tolist() == [3, 3, 7, 7]


def test_e4m3_encoder_edges():
    # types.tkv:154-191 with e4m3 parameters (bias 7, w 3, emax 15, sat 0x7E)
    cases = {0.0: 0x00, -0.0: 0x00, 0.5: 0x30, 1.0: 0x38, -1.0: 0xB8, 240.0: 0x77, 247.0: 0x77,
             248.0: 0x7E, 256.0: 0x7E, 300.0: 0x7E, 448.0: 0x7E, 1e9: 0x7E, -1e9: 0xFE,
             2.0 ** -6: 0x08, 7.6 * 2.0 ** -9: 0x07, 2.0 ** -9: 0x01, 2.0 ** -10: 0x00,
             1.5 * 2.0 ** -10: 0x01, float("nan"): 0x7F, float("inf"): 0x7F, float("-inf"): 0xFF}
    for v, b in cases.items():
        assert O.e4m3_encode(v) == b, (v, hex(O.e4m3_encode(v)), hex(b))


def test_e4m3_decoder_table():
    # types.tkv:193-226: normals are OCP E4M3; 0x7F/0xFF decode to +/-Inf
    # (f32_bits_to_f64 returns 2^129 for exponent 255); subnormals decode
    # to half the OCP value (the decoder uses 127 - bias - n, types.tkv:221).
    for v in range(256):
        d = O.e4m3_decode(v)
        e, m, s = (v >> 3) & 15, v & 7, -1.0 if v & 0x80 else 1.0
        if e == 15 and m == 7:
            assert math.isinf(d) and math.copysign(1, d) == s
        elif e == 0:
            assert d == s * m * 2.0 ** -10
        else:
            assert d == s * (1 + m / 8) * 2.0 ** (e - 7)


def test_rne_rshift():
    assert O.rne_rshift(0b1010, 2) == 2      # 2.5 -> 2
    assert O.rne_rshift(0b1110, 2) == 4      # 3.5 -> 4
    assert O.rne_rshift(0b1011, 2) == 3      # 2.75 -> 3
    assert O.rne_rshift(5, 0) == 5
    assert O.rne_rshift(1 << 30, 41) == 0


def test_f64_to_f32_bits_matches_ieee():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32),
                        (rng.standard_normal(200) * 1e-40).astype(np.float32),
                        np.array([np.finfo(np.float32).max, np.finfo(np.float32).tiny, 3e-45], np.float32)])
    for v in x:
        if v == 0 or abs(v) == np.float32(1e-45):
            continue
        assert O.f64_to_f32_bits(float(v)) == int(np.float32(v).view(np.uint32)), v
    assert O.f64_to_f32_bits(-0.0) == 0
    # f32_bits.tkv:37-39 returns the sign only when sh = e + 149 <= 0, so the
    # smallest subnormal 2^-149 maps to zero (restated as written)
    assert O.f64_to_f32_bits(2.0 ** -149) == 0


def test_quantize_ties_half_even_and_floors():
    # x*inv exactly on .5 -> round half to even (Math.Round)
    x = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, 127.5, -300.0], np.float32)
    assert O.quantize_int8_symmetric(x, 1.0).tolist() == [0, 2, 2, 0, -2, -2, 126, 127, -127]
    # scale <= 1e-8 -> inv = 1/1e-8 (engine.tkv:219-222)
    assert O.quantize_int8_symmetric(np.array([1e-9, -2e-8], np.float32), 0.0).tolist() == [0, -2]
    # per-channel floor, engine.tkv:244-245
    q = O.quantize_int8_per_channel(np.array([[1e-9, 3e-8]], np.float32), 1, 2, np.array([0.0], np.float32))
    assert q.tolist() == [[0, 3]]
    # calibrate floor: all-zero data -> scale = fl32(1e-8/127)
    p = O.calibrate_minmax(np.zeros(16, np.float32))
    assert p.scale == np.float32(1e-8 / 127.0)
    # empty data -> identity params (engine.tkv:9-15)
    p = O.calibrate_minmax(np.zeros(0, np.float32))
    assert p.scale == 1.0 and p.zero_point == 0


def test_quantize_nan_inf():
    x = np.array([np.nan, np.inf, -np.inf], np.float32)
    assert O.quantize_int8_symmetric(x, 0.5).tolist() == [0, 127, -127]


def test_calibrate_asymmetric():
    # engine.tkv:31-36
    p = O.calibrate_minmax(np.array([0.0, 1.0, 2.0], np.float32), 0)
    assert abs(p.scale - 2.0 / 255.0) < 1e-9 and p.zero_point == -128


def test_per_channel_value_errors():
    with pytest.raises(ValueError):
        O.calibrate_per_channel_minmax(np.zeros(4, np.float32), 0, 4)
    with pytest.raises(ValueError):
        O.calibrate_per_channel_minmax(np.zeros(4, np.float32), 2, 4)
    with pytest.raises(ValueError):
        O.matmul_int8_per_channel(np.zeros((2, 4), np.int8), np.zeros((3, 4), np.int8), None, 1.0,
                                  np.ones(2, np.float32))


def test_dot_int8_unrolled_tail():
    rng = np.random.default_rng(1)
    for k in [1, 31, 32, 33, 63, 64, 100, 768]:
        a = rng.integers(-127, 128, k).astype(np.int8)
        b = rng.integers(-127, 128, k).astype(np.int8)
        assert O.dot_int8(a, b) == int(np.dot(a.astype(np.int64), b.astype(np.int64)))


def test_gemm_epilogue_f64_model():
    rng = np.random.default_rng(2)
    m, n, k = 7, 9, 70
    A = rng.integers(-127, 128, (m, k)).astype(np.int8)
    W = rng.integers(-127, 128, (n, k)).astype(np.int8)
    bias = rng.standard_normal(n).astype(np.float32)
    sa = np.float32(0.0123)
    sw = (rng.random(n) * 0.01).astype(np.float32)
    Y = O.matmul_int8_per_channel(A, W, bias, sa, sw)
    acc = A.astype(np.int64) @ W.astype(np.int64).T
    ref = ((acc.astype(np.float64) * np.float64(sa)) * sw.astype(np.float64) + bias.astype(np.float64))
    assert np.array_equal(Y, ref.astype(np.float32))
    Ys = O.matmul_int8_symmetric(A, W, None, sa, np.float32(0.5))
    s = np.float64(sa) * np.float64(np.float32(0.5))
    assert np.array_equal(Ys, (acc.astype(np.float64) * s).astype(np.float32))


def test_fp8_gemm_exact_f64_sum():
    rng = np.random.default_rng(3)
    A = rng.integers(0, 256, (5, 40)).astype(np.uint8)
    W = rng.integers(0, 256, (6, 40)).astype(np.uint8)
    A[(A & 0x7F) == 0x7F] = 0x10
    W[(W & 0x7F) == 0x7F] = 0x10
    Y = O.matmul_fp8_e4m3(A, W, None)
    da = O.dequantize_fp8_e4m3(A).astype(np.float64)
    dw = O.dequantize_fp8_e4m3(W).astype(np.float64)
    assert np.array_equal(Y, (da @ dw.T).astype(np.float32))


def test_gelu_definitions():
    # A-S 7.1.26 erf is within 1.5e-7 of erf
    for x in np.linspace(-6, 6, 101):
        assert abs(O.erf_as(float(x)) - math.erf(float(np.float32(x)))) < 3e-7
    assert abs(O.gelu_erf(1.0) - 0.8413447) < 1e-6
    assert abs(O.gelu_tanh(1.0) - 0.8411920) < 1e-6


def test_gi_noise_generator():
    # gpt2_ref.tkv:1977-1991: deterministic, N(0, 0.02)
    a = O.gi_noise(20000, 11)
    assert np.array_equal(a, O.gi_noise(20000, 11))
    assert abs(a.mean()) < 1e-3 and abs(a.std() - 0.02) < 1e-3


def _g2_forward_fp32_linears(d):
    """Reduced GPT-2 of the fixtures through the oracle glue, with the
    fixtures' fp32 Conv1D linears done in f64 (gpt2_ref.tkv:91-117)."""
    V, H, NH, L = 256, 64, 4, 2
    ids, pos = d["ids"], d["pos"]
    T = ids.size
    wte = d["w_wte"].reshape(V, H)
    x = O.embed(ids, pos, wte, d["w_wpe"].reshape(-1, H))
    hs = [x]

    def lin(x, w, b):
        return (x.astype(np.float64) @ w.astype(np.float64) + b).astype(np.float32)

    for i in range(L):
        a = O.layernorm(x, d[f"w_ln1_g{i}"], d[f"w_ln1_b{i}"])
        qkv = lin(a, d[f"w_attn_w{i}"].reshape(H, 3 * H), d[f"w_attn_b{i}"])
        ctx = O.attention_causal(qkv, NH, [0, T])
        r = O.add(x, lin(ctx, d[f"w_proj_w{i}"].reshape(H, H), d[f"w_proj_b{i}"]))
        m = O.layernorm(r, d[f"w_ln2_g{i}"], d[f"w_ln2_b{i}"])
        f = O.gelu_erf_array(lin(m, d[f"w_mlp_w1{i}"].reshape(H, 4 * H), d[f"w_mlp_b1{i}"]))
        x = O.add(r, lin(f, d[f"w_mlp_w2{i}"].reshape(4 * H, H), d[f"w_mlp_b2{i}"]))
        hs.append(x)
    xf = O.layernorm(x, d["w_lnf_g"], d["w_lnf_b"])
    return hs, O.lm_head(xf, wte)


def test_gpt2_glue_matches_reference_fixtures():
    d = np.load(GOLDEN)
    hs, logits = _g2_forward_fp32_linears(d)
    for i in range(3):
        assert np.abs(hs[i].ravel() - d[f"h{i}"]).max() < 1e-6
    assert np.abs(logits.ravel() - d["logits"]).max() < 1e-5
    lg = logits.astype(np.float64)
    ids = d["ids"]
    lse = np.log(np.exp(lg).sum(1))
    loss = np.mean(lse - lg[np.arange(ids.size), ids])
    assert abs(loss - float(d["loss"][0])) < 1e-5


def test_f32_quotient_by_127_equals_binary64_rounded():
    """calibrate_per_channel_minmax's scale fl32(fl64(amax) / 127) equals the
    correctly rounded f32 quotient (the per-channel quantizer forms it so):
    an f64 quotient by 127 repeats a 7-bit pattern and never lands on an f32
    rounding midpoint.  Every 251st positive finite binary32 here (checked
    on all 2^31 - 2^23 of them once, no mismatch)."""
    bits = np.arange(1, 0x7F800000, 251, dtype=np.uint64).astype(np.uint32)
    a = bits.view(np.float32)
    ref = (a.astype(np.float64) / 127.0).astype(np.float32)
    assert np.array_equal(ref.view(np.uint32), (a / np.float32(127.0)).view(np.uint32))
