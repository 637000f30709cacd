"""CPU checks of the INT4 oracle (tv/quantization/int4.tkv restated in
oracle/tvq_oracle.c): the reference's own test (inference_tests.tkv:634-656)
as written, the cases its comments derive by hand (int4.tkv:96-135), and a
second, pure-Python restatement of the reference's loops (f64 locals, f32
list stores) on seeded inputs."""
import numpy as np
import pytest

import oracle as O


def _f32(v):
    return float(np.float32(v))


def _round_half_even(v):
    return int(np.rint(v))


def py_quantize_int4_grouped(src, rows, cols, gs):
    """int4.tkv:18-48 as written (f64 locals, f32 list stores)."""
    ng = cols // gs
    scales = []
    for r in range(rows):
        for g in range(ng):
            am = 0.0
            for c in range(gs):
                a = abs(float(src[r * cols + g * gs + c]))
                if a > am:
                    am = a
            if am < 0.00000001:
                am = 0.00000001
            scales.append(_f32(am / 7.0))
    packed = []
    for r in range(rows):
        for c in range(0, cols, 2):
            sc = scales[r * ng + c // gs]
            inv = 1.0 / sc
            q0 = max(-8, min(7, _round_half_even(float(src[r * cols + c]) * inv))) + 8
            q1 = max(-8, min(7, _round_half_even(float(src[r * cols + c + 1]) * inv))) + 8
            packed.append((q1 << 4) | q0)
    return np.array(packed, np.uint8), np.array(scales, np.float32)


def py_quantize_int4_grouped_asym(src, rows, cols, gs):
    """int4.tkv:68-150 as written."""
    ng = cols // gs
    scales, zps = [], []
    for r in range(rows):
        for gg in range(ng):
            mn = float(src[r * cols + gg * gs])
            mx = mn
            for c in range(1, gs):
                v = float(src[r * cols + gg * gs + c])
                if v < mn:
                    mn = v
                if v > mx:
                    mx = v
            if mx - mn < 0.00000001:
                mx = mn + 0.00000001
            sc = (mx - mn) / 15.0
            zp = _round_half_even(-mn / sc)
            zp = min(max(zp, 0), 15)
            if zp == 0:
                if mn > 0:
                    sc = mx / 15.0
                    if sc < 0.00000001:
                        sc = 0.00000001
                    zp = 0
            elif zp == 15:
                sc = -mn / 15.0
            if sc < 0.00000001:
                sc = 0.00000001
            scales.append(_f32(sc))
            zps.append(zp)
    packed = []
    for r in range(rows):
        for c in range(0, cols, 2):
            sc = scales[r * ng + c // gs]
            zp = zps[r * ng + c // gs]
            mn = -zp * sc
            q0 = max(0, min(15, _round_half_even((float(src[r * cols + c]) - mn) / sc)))
            q1 = max(0, min(15, _round_half_even((float(src[r * cols + c + 1]) - mn) / sc)))
            packed.append((q1 << 4) | q0)
    return np.array(packed, np.uint8), np.array(scales, np.float32), np.array(zps, np.int64)


def py_matmul_int4_grouped(A, packed, bias, m, n, k, gs, scales, perm=None):
    """int4.tkv:187-239 as written (f64 accumulation, one f32 store)."""
    ng = k // gs
    y = np.empty(m * n, np.float32)
    for mm in range(m):
        for nn in range(n):
            acc = 0.0
            for kk in range(k):
                b = int(packed[nn * (k // 2) + kk // 2])
                nib = (b & 0xF) if kk % 2 == 0 else ((b >> 4) & 0xF)
                w = float(nib - 8) * float(scales[nn * ng + kk // gs])
                acc = acc + float(A[mm * k + (perm[kk] if perm is not None else kk)]) * w
            y[mm * n + nn] = _f32(acc + (float(bias[nn]) if len(bias) else 0.0))
    return y


def test_reference_test_awq_asym_and_permute():
    # tv/tests/inference_tests.tkv:634-656
    w = np.array([float(i) - 2.0 for i in range(8)], np.float32)
    packed, scales, zps = O.quantize_int4_grouped_asym(w, 1, 8, 4)
    assert packed.size == 4 and scales.size == 2 and zps.size == 2
    y = O.dequantize_int4_grouped_asym(packed, 1, 8, 4, scales, zps).ravel()
    assert np.all(np.abs(w - y) < scales.max() * 2.0)
    p = np.zeros(6, np.float32)
    q = O.permute_cols(O.permute_cols(p, 2, 3, [2, 0, 1]), 2, 3, [2, 0, 1], inverse=True)
    assert np.array_equal(q.ravel(), p)


def test_reference_comment_cases():
    # int4.tkv:96-112: an all-positive group [2, 3, 4, 5] round-trips
    # exactly (zp 0, scale max/15); [4, 5, 6, 7] keeps every value within
    # half a step (the earlier code sent 4.0 to 2.667)
    w = np.array([2, 3, 4, 5, 4, 5, 6, 7], np.float32)
    packed, scales, zps = O.quantize_int4_grouped_asym(w, 1, 8, 4)
    assert zps.ravel().tolist() == [0, 0]
    y = O.dequantize_int4_grouped_asym(packed, 1, 8, 4, scales, zps).ravel()
    assert np.array_equal(y[:4], w[:4])
    assert np.all(np.abs(y[4:] - w[4:]) <= scales.ravel()[1] / 2 + 1e-6)
    # an all-negative group clamps zp to 15 with scale -min/15
    w = np.array([-5, -4, -3, -2], np.float32)
    packed, scales, zps = O.quantize_int4_grouped_asym(w, 1, 4, 4)
    assert zps.ravel()[0] == 15 and scales.ravel()[0] == np.float32(5.0 / 15.0)
    # symmetric: scale max|x|/7, nibbles biased by 8, low nibble first
    w = np.array([7.0, -7.0, 3.5, 0.0], np.float32)
    packed, scales = O.quantize_int4_grouped(w, 1, 4, 4)
    assert scales.ravel()[0] == 1.0
    assert packed.ravel().tolist() == [(1 << 4) | 15, (8 << 4) | 12]  # 3.5 -> 4 (half to even)
    # a constant zero group uses the 1e-8 floor
    packed, scales = O.quantize_int4_grouped(np.zeros(4, np.float32), 1, 4, 2)
    assert np.all(scales == np.float32(1e-8 / 7.0)) and np.all(packed == 0x88)


def test_shape_errors():
    x = np.zeros(12, np.float32)
    with pytest.raises(ValueError):
        O.quantize_int4_grouped(x, 1, 12, 5)      # cols not a multiple of group_size
    with pytest.raises(ValueError):
        O.quantize_int4_grouped(x[:9], 1, 9, 3)   # odd cols
    with pytest.raises(ValueError):
        O.permute_cols(x, 3, 4, [0, 1, 2])        # perm length


@pytest.mark.parametrize("rows,cols,gs", [(3, 16, 4), (5, 64, 32), (2, 12, 6)])
def test_oracle_codecs_match_python_restatement(rows, cols, gs):
    rng = np.random.default_rng(rows * 100 + cols)
    x = (rng.standard_normal(rows * cols) * rng.choice([0.01, 1.0, 50.0], rows * cols)).astype(np.float32)
    x[::7] = np.round(x[::7] * 2) / 2  # exact halves: ties
    pk, sc = O.quantize_int4_grouped(x, rows, cols, gs)
    rpk, rsc = py_quantize_int4_grouped(x, rows, cols, gs)
    assert np.array_equal(pk.ravel(), rpk) and np.array_equal(sc.ravel().view(np.uint32), rsc.view(np.uint32))
    pk, sc, zp = O.quantize_int4_grouped_asym(x, rows, cols, gs)
    rpk, rsc, rzp = py_quantize_int4_grouped_asym(x, rows, cols, gs)
    assert np.array_equal(pk.ravel(), rpk) and np.array_equal(zp.ravel(), rzp)
    assert np.array_equal(sc.ravel().view(np.uint32), rsc.view(np.uint32))


@pytest.mark.parametrize("with_perm", [False, True])
def test_oracle_matmul_matches_python_restatement(with_perm):
    rng = np.random.default_rng(5)
    m, n, k, gs = 3, 5, 32, 8
    A = rng.standard_normal(m * k).astype(np.float32)
    W = rng.standard_normal(n * k).astype(np.float32)
    pk, sc = O.quantize_int4_grouped(W, n, k, gs)
    bias = rng.standard_normal(n).astype(np.float32)
    perm = rng.permutation(k).astype(np.int64) if with_perm else None
    y = O.matmul_int4_grouped(A.reshape(m, k), pk.reshape(n, k // 2), bias, gs, sc, perm).ravel()
    ref = py_matmul_int4_grouped(A, pk.ravel(), bias, m, n, k, gs, sc.ravel(), perm)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
    # act order: gathering A's columns equals permuting them first
    if with_perm:
        Ap = O.permute_cols(A, m, k, perm)
        y2 = O.matmul_int4_grouped(Ap.reshape(m, k), pk.reshape(n, k // 2), bias, gs, sc).ravel()
        assert np.array_equal(y, y2)
