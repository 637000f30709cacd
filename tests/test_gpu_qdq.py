"""GPU parity of the ONNX QDQ operator family (tv/runtime/session.tkv:
1896-2071, 2789-2905) against the oracle, bit-exact: quantize / dequantize
per tensor and per axis with zero points, exact ties, NaN / Inf, the 1e-12
scale floor; MatMulInteger and QLinearMatMul on the tcgen05 INT8 GEMM with
ragged K (the padded operand path) and zero points; DynamicQuantizeLinear; and
the runtime mirror running the reference's own operator tests
(tv/tests/inference_tests.tkv:903-938)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import _native as N
from tokenvector.inference_b200.runtime import session as RS

pytestmark = pytest.mark.gpu


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _quant(x, sc, zp=0, axis=1):
    x = np.ascontiguousarray(x, np.float32)
    sc = np.ascontiguousarray(np.atleast_1d(sc), np.float32)
    outer, dim, inner = O._axis_split(x.shape, axis, sc.size)
    y = np.empty(x.shape, np.int8)
    N.call("tvq_quantize_linear", _p(x), _p(y), outer, dim, inner, _p(sc), sc.size, zp)
    return y


def _dequant(x, sc, zp=0, axis=1):
    x = np.ascontiguousarray(x, np.int8)
    sc = np.ascontiguousarray(np.atleast_1d(sc), np.float32)
    outer, dim, inner = O._axis_split(x.shape, axis, sc.size)
    y = np.empty(x.shape, np.float32)
    N.call("tvq_dequantize_linear", _p(x), _p(y), outer, dim, inner, _p(sc), sc.size, zp)
    return y


@pytest.mark.parametrize("shape,axis,nsc", [((1000003,), 0, 1), ((64, 768), 1, 768), ((3, 50, 7), 1, 50),
                                            ((4, 6, 5), -1, 5), ((37,), 0, 1)])
@pytest.mark.parametrize("zp", [0, -7, 120])
def test_quantize_dequantize_linear_bit_exact(shape, axis, nsc, zp):
    rng = np.random.default_rng(sum(shape) + zp)
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    sc = (rng.random(nsc) * 0.05 + 0.001).astype(np.float32)
    # exact ties at half-integers (power-of-two scales), specials
    flat = x.reshape(-1)
    t = min(64, flat.size)
    flat[:t] = ((np.arange(64) - 32 + 0.5).astype(np.float32) * 0.25)[:t]
    if nsc == 1:
        sc[0] = 0.25
        if flat.size >= 70:
            flat[64:70] = [np.nan, np.inf, -np.inf, 0.0, -0.0, 1e30]
    q = _quant(x, sc, zp, axis)
    assert np.array_equal(q, O.quantize_linear(x, sc, zp, axis))
    d = _dequant(q, sc, zp, axis)
    assert np.array_equal(d.view(np.int32), O.dequantize_linear(q, sc, zp, axis).view(np.int32))


def test_quantize_linear_scale_floor_and_large_zero_point():
    x = np.array([1e-11, -1e-13, 0.0, 1e-9, 2.5e-12, -3.5e-12], np.float32)
    for sc in ([0.0], [1e-13], [-1.0], [np.nan]):
        assert np.array_equal(_quant(x, sc), O.quantize_linear(x, sc))
    for zp in (300, -300, 1 << 40):
        assert np.array_equal(_quant(x * 1e12, [1.0], zp), O.quantize_linear(x * 1e12, [1.0], zp))
    d = _dequant(np.array([-128, 127, 0], np.int8), [3.0], 1 << 30)
    assert np.array_equal(d, O.dequantize_linear(np.array([-128, 127, 0], np.int8), [3.0], 1 << 30))


@pytest.mark.parametrize("m,k,n", [(2, 2, 2), (1, 768, 3072), (130, 77, 300), (1024, 768, 2304), (5, 1, 17)])
def test_matmul_integer_bit_exact(m, k, n):
    rng = np.random.default_rng(m + k + n)
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (k, n), dtype=np.int8)
    y = np.empty((m, n), np.int32)
    N.call("tvq_matmul_integer", _p(a), _p(b), _p(y), m, k, n)
    assert np.array_equal(y, O.matmul_integer(a, b))


@pytest.mark.parametrize("m,k,n", [(1, 64, 64), (130, 77, 300), (512, 768, 768)])
@pytest.mark.parametrize("zps", [(0, 0, 0), (3, -5, 7), (-128, 127, -20)])
def test_qlinear_matmul_bit_exact(m, k, n, zps):
    rng = np.random.default_rng(m * 7 + k + n)
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (k, n), dtype=np.int8)
    zpa, zpb, zpy = zps
    sa, sb = np.float32(0.02), np.float32(0.013)
    sy = np.float32(float(sa) * float(sb) * np.sqrt(k) * 40)
    y = np.empty((m, n), np.int8)
    N.call("tvq_qlinear_matmul", _p(a), float(sa), zpa, _p(b), float(sb), zpb, float(sy), zpy, _p(y), m, k, n)
    assert np.array_equal(y, O.qlinear_matmul(a, sa, zpa, b, sb, zpb, sy, zpy))


def test_qlinear_matmul_ties_and_zero_scale():
    # products landing exactly on half-integers take the binary64 path
    a = np.array([[1, 3, 5, -1, -3]], np.int8).T.copy()   # [5, 1]
    b = np.ones((1, 4), np.int8)
    for sy in (0.0, 2.0):
        y = np.empty((5, 4), np.int8)
        N.call("tvq_qlinear_matmul", _p(a), 0.5, 0, _p(b), 1.0, 0, sy, 0, _p(y), 5, 1, 4)
        assert np.array_equal(y, O.qlinear_matmul(a, 0.5, 0, b, 1.0, 0, sy, 0))


@pytest.mark.parametrize("n", [1, 3, 5, 1000, 1 << 20])
def test_dynamic_quantize_linear_bit_exact(n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 2 + 0.3).astype(np.float32)
    if n == 3:
        x[:] = [0.0, 1.0, 2.0]
    cases = [x]
    if n == 1000:
        cases += [np.abs(x), -np.abs(x), np.zeros(n, np.float32), np.where(np.arange(n) % 7 == 0, np.nan, x)
                  .astype(np.float32)]
        bad = x.copy()
        bad[0] = np.nan
        cases.append(bad)
    for c in cases:
        y = np.empty(n, np.int8)
        s = np.zeros(1, np.float32)
        z = np.zeros(1, np.float32)
        N.call("tvq_dynamic_quantize_linear", _p(c), n, _p(y), _p(s), _p(z))
        ry, rs, rz = O.dynamic_quantize_linear(c)
        assert np.array_equal(y, ry)
        assert (np.isnan(s[0]) and np.isnan(rs)) or s[0] == np.float32(rs)
        assert z[0] == rz


def test_runtime_mirror_reference_operator_tests():
    # inference_tests.tkv:903-921 -- MatMulInteger through the graph executor
    g = RS.ExecutionGraph()
    g.inputs, g.outputs = ["A", "B"], ["Y"]
    g.get_or_create_tensor("A", [2, 2], RS.TensorDataType_Int8)
    g.get_or_create_tensor("B", [2, 2], RS.TensorDataType_Int8)
    g.get_or_create_tensor("Y", [2, 2], RS.TensorDataType_Int32)
    nd = RS.new_node("m", RS.OperatorType_MatMulInteger)
    nd.inputs, nd.outputs = ["A", "B"], ["Y"]
    g.nodes.append(nd)
    s = RS.session_from_graph(g, 0)
    yo = np.zeros(4, np.int32)
    s.run([RS.named_qdata("A", np.array([1, 2, 3, 4], np.int8)), RS.named_qdata("B", np.ones(4, np.int8))],
          [RS.named_idata("Y", yo)])
    s.close()
    assert yo.tolist() == [3, 3, 7, 7]
    # inference_tests.tkv:923-938 -- DynamicQuantizeLinear with scale / zero-point outputs
    g = RS.ExecutionGraph()
    g.inputs, g.outputs = ["I0"], ["Y", "YS", "YZ"]
    g.get_or_create_tensor("I0", [3])
    g.get_or_create_tensor("Y", [3], RS.TensorDataType_Int8)
    g.get_or_create_tensor("YS", [1])
    g.get_or_create_tensor("YZ", [1])
    nd = RS.new_node("q", RS.OperatorType_DynamicQuantizeLinear)
    nd.inputs, nd.outputs = ["I0"], ["Y", "YS", "YZ"]
    g.nodes.append(nd)
    s = RS.session_from_graph(g, 0)
    yq = np.zeros(3, np.int8)
    ysc = np.zeros(1, np.float32)
    yzp = np.zeros(1, np.float32)
    s.run([RS.named_tensor("I0", np.array([0.0, 1.0, 2.0], np.float32))],
          [RS.named_qdata("Y", yq), RS.named_tensor("YS", ysc), RS.named_tensor("YZ", yzp)])
    s.close()
    assert abs(ysc[0] - 2.0 / 255.0) < 1e-6 and yzp[0] == 0.0 and yq[0] == -128 and yq[2] == 127


def test_runtime_mirror_qdq_chain_and_fold():
    """QuantizeLinear (per axis) -> QLinearMatMul -> DequantizeLinear through
    the mirror, bit-exact against the oracle composition; with
    apply_optimizations a Q -> DQ pair is folded away."""
    rng = np.random.default_rng(3)
    m, k, n = 33, 48, 20
    x = rng.standard_normal((m, k)).astype(np.float32)
    bq = rng.integers(-128, 128, (k, n), dtype=np.int8)
    g = RS.ExecutionGraph()
    g.inputs, g.outputs = ["X"], ["Y"]
    g.get_or_create_tensor("X", [m, k])
    g.get_or_create_tensor("XQ", [m, k], RS.TensorDataType_Int8)
    g.get_or_create_tensor("B", [k, n], RS.TensorDataType_Int8)
    g.get_or_create_tensor("YQ", [m, n], RS.TensorDataType_Int8)
    g.get_or_create_tensor("Y", [m, n])
    scalars = {"XS": 0.02, "XZ": 2.0, "BS": 0.01, "BZ": -1.0, "YS": 0.05, "YZ": 4.0}
    for nm, v in scalars.items():
        g.get_or_create_tensor(nm, [1])
        g.initializers[nm] = [v]
    g.initializers_int8["B"] = bq.ravel()
    q = RS.new_node("q", RS.OperatorType_QuantizeLinear)
    q.inputs, q.outputs = ["X", "XS", "XZ"], ["XQ"]
    mm = RS.new_node("mm", RS.OperatorType_QLinearMatMul)
    mm.inputs, mm.outputs = ["XQ", "XS", "XZ", "B", "BS", "BZ", "YS", "YZ"], ["YQ"]
    dq = RS.new_node("dq", RS.OperatorType_DequantizeLinear)
    dq.inputs, dq.outputs = ["YQ", "YS", "YZ"], ["Y"]
    g.nodes = [q, mm, dq]
    s = RS.session_from_graph(g, 1)  # nothing to fold: Q feeds QLinearMatMul
    assert len(g.nodes) == 3
    y = s.run_single(x.ravel(), "X", "Y")
    s.close()
    xq = O.quantize_linear(x, [0.02], 2)
    yq = O.qlinear_matmul(xq, 0.02, 2, bq, 0.01, -1, 0.05, 4)
    ref = O.dequantize_linear(yq, [0.05], 4)
    assert np.array_equal(y.reshape(m, n), ref)
