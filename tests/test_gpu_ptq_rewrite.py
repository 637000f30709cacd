"""The PTQ rewrite end to end on the GPU: an fp32 graph (MatMul + Add [+ Relu |
Gelu], the shape OperatorFusionPass folds, tv/runtime/session.tkv:3698-3771)
quantized by PtqRewritePass and executed by InferenceSession, against the
oracle's restatement of the same PTQ recipe (engine.tkv:13-36, 202-250,
matmul.tkv:17-29, kernels.tkv:14-38)."""
import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import ptq
from tokenvector.inference_b200.runtime import session as R

pytestmark = pytest.mark.gpu


def _graph(m, k, n, w, bias, act_op=None):
    g = R.ExecutionGraph("lin")
    g.inputs.append("x")
    g.outputs.append("y")
    g.get_or_create_tensor("x", [m, k])
    g.get_or_create_tensor("W", list(w.shape))
    g.initializers["W"] = w.ravel().copy()
    g.get_or_create_tensor("b", [n])
    g.initializers["b"] = bias.copy()
    g.get_or_create_tensor("xw", [m, n])
    mm = R.new_node("fc", R.OperatorType_MatMul)
    mm.inputs, mm.outputs = ["x", "W"], ["xw"]
    add = R.new_node("fc_bias", R.OperatorType_Add)
    add.inputs, add.outputs = ["xw", "b"], ["xb" if act_op else "y"]
    g.nodes += [mm, add]
    if act_op:
        g.get_or_create_tensor("xb", [m, n])
        a = R.new_node("fc_act", act_op)
        a.inputs, a.outputs = ["xb"], ["y"]
        g.nodes.append(a)
    g.get_or_create_tensor("y", [m, n])
    return g


def _oracle(x, batches, w_nk, bias):
    n, k = w_nk.shape
    sa = O.calibrate_minmax(np.concatenate([b.ravel() for b in batches])).scale
    xq = O.quantize_int8_symmetric(x, sa)
    sw = O.per_channel_scales(w_nk, n, k)
    wq = O.quantize_int8_per_channel(w_nk, n, k, sw)
    return O.matmul_int8_per_channel(xq, wq, bias, np.float32(sa), sw), wq, sw, np.float32(sa)


def _run(g, x, m, n, ptq_pass):
    s = R.session_from_graph(g, 1, 0, ptq_pass)
    y = R.NamedTensor("y", data=np.zeros(m * n, np.float32))
    s.run([R.named_tensor("x", x.ravel())], [y])
    s.close()
    return y.data.reshape(m, n)


@pytest.mark.parametrize("m,k,n,trans_b", [(64, 256, 192, False), (130, 200, 300, True), (1024, 768, 3072, False)])
def test_rewritten_linear_bit_exact(m, k, n, trans_b):
    rng = np.random.default_rng(m + k)
    batches = [rng.standard_normal((m, k)).astype(np.float32) for _ in range(3)]
    x = batches[1]
    w_nk = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    g = _graph(m, k, n, w_nk if trans_b else np.ascontiguousarray(w_nk.T), bias)
    p = R.PtqRewritePass(calibration={"x": batches})
    y = _run(g, x, m, n, p)
    ref, wq, sw, sa = _oracle(x, batches, w_nk, bias)
    q = p.linears[0]
    assert np.array_equal(q.w, wq) and np.array_equal(q.scales_w.view(np.uint32), sw.view(np.uint32))
    assert np.float32(q.scale_a).view(np.uint32) == sa.view(np.uint32)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


def test_rewritten_linear_relu_fused_bit_exact():
    m, k, n = 96, 128, 160
    rng = np.random.default_rng(5)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w_nk = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.05).astype(np.float32)
    g = _graph(m, k, n, np.ascontiguousarray(w_nk.T), bias, R.OperatorType_Relu)
    y = _run(g, x, m, n, R.PtqRewritePass(calibration={"x": [x]}))
    ref = _oracle(x, [x], w_nk, bias)[0]
    assert np.array_equal(y.view(np.uint32), np.maximum(ref, np.float32(0)).view(np.uint32))


def test_rewritten_linear_gelu_fused():
    """GELU (tanh form) runs in the GEMM epilogue in the reference's binary64
    model with CUDA's exp; the oracle uses the host libm's exp.  Tolerance: 1
    ulp of the f32 result (a binary64 quotient within an ulp of an f32
    rounding boundary), and at most 1 % of the elements off at all."""
    m, k, n = 128, 256, 256
    rng = np.random.default_rng(6)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w_nk = (rng.standard_normal((n, k)) * 0.1).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    # a square weight is always read as [N, K] (_exec_linear tests shape[1] == k
    # first, session.tkv:756-761): store it that way
    g = _graph(m, k, n, w_nk, bias, R.OperatorType_Gelu)
    y = _run(g, x, m, n, R.PtqRewritePass(calibration={"x": [x]}))
    pre = _oracle(x, [x], w_nk, bias)[0]
    ref = np.array([O.gelu_tanh(float(v)) for v in pre.ravel()], np.float32).reshape(m, n)
    err = np.abs(y.astype(np.float64) - ref)
    tol = np.spacing(np.abs(ref)).astype(np.float64)
    assert (err <= tol).all(), float((err / tol).max())
    assert (err > 0).mean() < 0.01


def test_artefact_reload_reproduces_session(tmp_path):
    """Calibrate once, export, then rebuild from the artefact alone: the
    second session needs no calibration data and gives the same bits."""
    m, k, n = 256, 384, 512
    rng = np.random.default_rng(7)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    g1 = _graph(m, k, n, w, bias, R.OperatorType_Gelu)
    y1 = _run(g1, x, m, n, R.PtqRewritePass(calibration={"x": [x]}))
    path = str(tmp_path / "lin.tvqptq")
    assert R.export_ptq(g1, path) == 1
    g2 = _graph(m, k, n, w, bias, R.OperatorType_Gelu)
    y2 = _run(g2, x, m, n, R.PtqRewritePass(artefact=path))
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    assert ptq.load(path)[0][0].act == R.ActivationFunction_GELU
