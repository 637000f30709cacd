"""The ONNX QDQ operator family on the CPU oracle: the reference's own known
answers (tv/tests/inference_tests.tkv:903-938) and hand-derived cases of the
semantics restated from tv/runtime/session.tkv:1896-2071, 2789-2905; and the
QdqFoldPass graph rewrite of the runtime mirror (host logic)."""
import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200.runtime import session as RS


def test_matmul_integer_known_answer():
    # inference_tests.tkv:903-921: A = [[1, 2], [3, 4]], B = ones -> 3, 3, 7, 7
    y = O.matmul_integer(np.array([[1, 2], [3, 4]], np.int8), np.ones((2, 2), np.int8))
    assert y.tolist() == [[3, 3], [7, 7]]


def test_dynamic_quantize_linear_known_answer():
    # inference_tests.tkv:923-938: [0, 1, 2] -> scale 2/255, zero point 0, ends -128 / 127
    y, s, z = O.dynamic_quantize_linear(np.array([0.0, 1.0, 2.0], np.float32))
    assert abs(s - 2.0 / 255.0) < 1e-6 and z == 0.0
    assert y[0] == -128 and y[2] == 127


def test_dynamic_quantize_linear_semantics():
    # all positive: mn is clamped to 0 -> zp 0; all negative: mx -> 0, zp 255
    y, s, z = O.dynamic_quantize_linear(np.array([-4.0, -1.0], np.float32))
    assert z == 255.0 and abs(s - 4.0 / 255.0) < 1e-7 and y[0] == -128 and y[1] == 127 - 64
    # constant zero input: range floored at 1e-8
    y, s, z = O.dynamic_quantize_linear(np.zeros(5, np.float32))
    assert s == np.float32(1e-8 / 255.0) and z == 0.0 and (y == -128).all()
    # NaN first element: scale NaN, zero point 0, every output 0 - 128
    y, s, z = O.dynamic_quantize_linear(np.array([np.nan, 1.0, 2.0], np.float32))
    assert np.isnan(s) and z == 0.0 and (y == -128).all()


def test_quantize_linear_rounding_floor_zero_point_clamp():
    x = np.array([[0.5, 1.5, 2.5, -0.5, -1.5, 3.49, 400.0, -400.0]], np.float32)
    assert O.quantize_linear(x, [1.0]).tolist() == [[0, 2, 2, 0, -2, 3, 127, -128]]
    assert O.quantize_linear(x, [1.0], zero_point=10).tolist() == [[10, 12, 12, 10, 8, 13, 127, -128]]
    # scale floor 1e-12 (a double): 1e-11 / 1e-12 = 10, 1e-9 saturates
    assert O.quantize_linear(np.array([1e-11, -1e-13, 0.0, 1e-9], np.float32), [0.0]).tolist() == [10, 0, 0, 127]
    # NaN -> int() 0 -> zero point
    assert O.quantize_linear(np.array([np.nan], np.float32), [1.0], zero_point=3).tolist() == [3]


def test_quantize_dequantize_per_axis():
    x = np.arange(12, dtype=np.float32).reshape(2, 3, 2)
    sc = np.array([1.0, 2.0, 4.0], np.float32)
    q = O.quantize_linear(x, sc, axis=1)
    ref = np.rint(x / sc.reshape(1, 3, 1)).astype(np.int8)  # no ties here except the half-even ones below
    assert (q == ref).all()
    d = O.dequantize_linear(q, sc, zero_point=1, axis=1)
    assert np.array_equal(d, ((q.astype(np.int64) - 1) * sc.reshape(1, 3, 1)).astype(np.float32))
    with pytest.raises(ValueError):
        O.quantize_linear(x, [1.0, 2.0], axis=1)
    # negative axis counts from the end
    assert np.array_equal(O.quantize_linear(x, [1.0, 2.0], axis=-1), np.rint(x / np.array([1.0, 2.0], np.float32)))


def test_qlinear_matmul_hand_case():
    a = np.array([[1, 2], [3, 4]], np.int8)
    b = np.ones((2, 2), np.int8)
    # (a - 1) @ b = [[1, 1], [5, 5]]; * 0.5 * 2 / 0.25 = 4 -> [[4, 4], [20, 20]] + 3
    assert O.qlinear_matmul(a, 0.5, 1, b, 2.0, 0, 0.25, 3).tolist() == [[7, 7], [23, 23]]
    # scale_y 0 reads as 1; ties to even: acc 1 * 2.5 -> 2
    assert O.qlinear_matmul(np.array([[1]], np.int8), 2.5, 0, np.array([[1]], np.int8), 1.0, 0, 0.0, 0).tolist() == [[2]]
    # saturation
    assert O.qlinear_matmul(np.array([[100]], np.int8), 1.0, 0, np.array([[100]], np.int8), 1.0, 0, 1.0, 0).tolist() == [[127]]


def _qdq_graph():
    g = RS.ExecutionGraph()
    g.inputs = ["X"]
    g.outputs = ["Y"]
    for nm, shape in (("X", [4]), ("S", [1]), ("XQ", [4]), ("XD", [4]), ("Y", [4])):
        g.get_or_create_tensor(nm, shape, RS.TensorDataType_Int8 if nm == "XQ" else RS.TensorDataType_Float)
    q = RS.new_node("q", RS.OperatorType_QuantizeLinear)
    q.inputs, q.outputs = ["X", "S"], ["XQ"]
    d = RS.new_node("dq", RS.OperatorType_DequantizeLinear)
    d.inputs, d.outputs = ["XQ", "S"], ["XD"]
    i = RS.new_node("id", RS.OperatorType_Identity)
    i.inputs, i.outputs = ["XD"], ["Y"]
    g.nodes = [q, d, i]
    return g


def test_qdq_fold_pass():
    g = _qdq_graph()
    assert RS.QdqFoldPass(1).run(g) == 1
    assert [n.name for n in g.nodes] == ["id"] and g.nodes[0].inputs == ["X"]
    assert RS.QdqFoldPass(1).run(g) == 0
    # a DequantizeLinear that does not read the Quantize output is kept
    g = _qdq_graph()
    g.nodes[1].inputs = ["X2", "S"]
    assert RS.QdqFoldPass(1).run(g) == 0 and len(g.nodes) == 3
    # graph outputs are redirected too
    g = _qdq_graph()
    g.outputs = ["XD"]
    g.nodes = g.nodes[:2]
    RS.QdqFoldPass(1).run(g)
    assert g.outputs == ["X"] and g.nodes == []


# ---- calibration methods (engine.tkv:42-197) on the oracle
def _outlier_data(n=50000, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    x[rng.choice(n, n // 1000, replace=False)] *= 20  # 0.1 % outliers x20 (BASELINE config 3's distribution)
    return x


def test_calibrate_kl_properties():
    x = _outlier_data()
    p = O.calibrate_kl(x)
    am = float(np.abs(x).max())
    thr = p.max_val
    assert p.zero_point == 0 and p.min_val == -thr
    # the threshold is a candidate: th * am / 2048 with th = 128 + 16 j
    th = thr / (am / 2048)
    assert abs(th - round(th)) < 1e-3 and (round(th) - 128) % 16 == 0 and 128 <= round(th) <= 2048
    assert thr < am  # outliers are clipped
    assert np.float32(thr / 127.0) == np.float32(p.scale)
    # tiny data -> calibrate_minmax(data, 1)
    t = np.array([1e-9, -2e-9], np.float32)
    q, r = O.calibrate_kl(t), O.calibrate_minmax(t, 1)
    assert (q.scale, q.max_val) == (r.scale, r.max_val)
    assert O.calibrate_kl(np.zeros(0, np.float32)).scale == 1.0


def test_calibrate_percentile_semantics():
    x = _outlier_data()
    ab = np.sort(np.abs(x))
    for pct in (99.99, 99.0, 50.0, 100.0, 0.001):
        idx = int(min(len(x) - 1, float(np.float32(pct)) / 100.0 * len(x)))
        p = O.calibrate_percentile(x, pct)
        assert p.max_val == ab[idx] and p.scale == np.float32(float(ab[idx]) / 127.0)
    with pytest.raises(ValueError):
        O.calibrate_percentile(x, 0.0)
    with pytest.raises(ValueError):
        O.calibrate_percentile(x, 100.5)
    # asymmetric: data[0] enters unclamped
    y = np.array([50.0, 1.0, -1.0, 2.0], np.float32)
    p = O.calibrate_percentile(y, 50.0, 0)  # clip = the 2nd smallest |y| = 1.0
    assert p.max_val == 50.0 and p.min_val == -1.0


def test_calibrate_mse_properties():
    x = _outlier_data(20000, 3)
    p = O.calibrate_mse(x)
    curve = O.calibrate_mse_curve(x)
    c = int(np.argmin(curve)) + 1
    am = float(np.abs(x).max())
    assert p.max_val == np.float32(am * c / 50)
    assert O.calibrate_mse(x, 2).max_val == O.calibrate_mse(x, 4).max_val  # at least 4 candidates
