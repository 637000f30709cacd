"""The reference-facing graph API (mirror of tv/runtime/session.tkv) running
QuantizedGemm nodes on the GPU, built the way the reference's tests build
graphs (tv/tests/inference_tests.tkv:895-921)."""
import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200.runtime import session as R

pytestmark = pytest.mark.gpu


def _qgemm_graph(m, n, k, wq, bias, scale_a, scales_w=None, scale_b=1.0):
    g = R.ExecutionGraph("q")
    g.inputs.append("A")
    g.outputs.append("Y")
    g.get_or_create_tensor("A", [m, k], R.TensorDataType_Int8)
    g.get_or_create_tensor("W", [n, k], R.TensorDataType_Int8)
    g.get_or_create_tensor("Y", [m, n], R.TensorDataType_Float)
    g.initializers_int8["W"] = wq
    node = R.new_node("qg", R.OperatorType_QuantizedGemm)
    node.inputs += ["A", "W"]
    if bias is not None:
        g.get_or_create_tensor("B", [n], R.TensorDataType_Float)
        g.initializers["B"] = bias
        node.inputs.append("B")
    node.outputs.append("Y")
    node.scale_a = float(scale_a)
    node.scale_b = float(scale_b)
    node.scales_w = list(scales_w) if scales_w is not None else []
    node.activation = R.ActivationFunction_GELU  # ignored by QuantizedGemm, session.tkv:678-697
    g.nodes.append(node)
    return g


def test_matmul_integer_known_answer_through_quantized_gemm():
    # inference_tests.tkv:895-921: [[1,2],[3,4]] . ones -> 3,3,7,7
    g = _qgemm_graph(2, 2, 2, np.ones(4, np.int32), None, 1.0, scale_b=1.0)
    s = R.session_from_graph(g, 0)
    y = R.NamedTensor("Y", data=np.zeros(4, np.float32))
    s.run([R.named_qdata("A", np.array([1, 2, 3, 4], np.int32))], [y])
    assert y.data.tolist() == [3.0, 3.0, 7.0, 7.0]
    s.close()


@pytest.mark.parametrize("m,n,k", [(1, 64, 768), (16, 256, 256), (130, 300, 200), (1024, 768, 3072)])
def test_quantized_gemm_node_per_channel_bit_exact(m, n, k):
    rng = np.random.default_rng(m + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    sa = O.calibrate_minmax(x).scale
    xq = O.quantize_int8_symmetric(x, sa)
    sw = O.per_channel_scales(w, n, k)
    wq = O.quantize_int8_per_channel(w, n, k, sw)
    g = _qgemm_graph(m, n, k, wq.astype(np.int32), bias, sa, sw)   # list[i32] storage as the reference
    s = R.InferenceSession(g, 1)
    y = R.NamedTensor("Y", data=np.zeros(m * n, np.float32))
    s.run([R.named_qdata("A", xq.astype(np.int32))], [y])
    ref = O.matmul_int8_per_channel(xq, wq, bias, np.float32(sa), sw)
    assert np.array_equal(y.data.reshape(m, n).view(np.uint32), ref.view(np.uint32))
    s.close()
    with pytest.raises(R.Disposed):
        s.run([], [])


def test_quantized_gemm_node_symmetric_and_run_single():
    rng = np.random.default_rng(9)
    m, n, k = 1, 40, 64
    wq = rng.integers(-127, 128, (n, k)).astype(np.int8)
    g = _qgemm_graph(m, n, k, wq, None, 0.02, None, scale_b=0.005)
    s = R.session_from_graph(g, 1)
    a = rng.integers(-127, 128, k).astype(np.int8)
    y = R.NamedTensor("Y", data=np.zeros(n, np.float32))
    s.run([R.named_qdata("A", a)], [y])
    ref = O.matmul_int8_symmetric(a.reshape(1, k), wq, None, np.float32(0.02), np.float32(0.005))
    assert np.array_equal(y.data.view(np.uint32), ref.ravel().view(np.uint32))


def test_scales_w_smaller_than_n_raises():
    g = _qgemm_graph(2, 3, 16, np.zeros(48, np.int8), None, 1.0, [1.0, 1.0])
    with pytest.raises(ValueError):
        R.InferenceSession(g, 1)
