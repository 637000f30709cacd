"""Graph passes of the PTQ path on the host: OperatorFusionPass (mirror of
tv/runtime/session.tkv:3698-3771) and the FusedLinear -> QuantizeInt8Symmetric
+ QuantizedGemm rewrite, driven by a PTQ artefact (no calibration, no GPU)."""
import numpy as np
import pytest

from tokenvector.inference_b200 import ptq
from tokenvector.inference_b200.runtime import session as R


def _linear_graph(m, k, n, act_op=None, trans_b=False, bias_init=True, x_shape=None):
    """x [m, k] -> MatMul (W [k, n], or [n, k] when trans_b) -> Add (bias) [-> act_op] -> y"""
    rng = np.random.default_rng(m * 7 + n)
    g = R.ExecutionGraph("lin")
    g.inputs.append("x")
    g.outputs.append("y")
    g.get_or_create_tensor("x", x_shape or [m, k])
    w = (rng.standard_normal((n, k) if trans_b else (k, n)) * 0.02).astype(np.float32)
    g.get_or_create_tensor("W", list(w.shape))
    g.initializers["W"] = w.ravel()
    g.get_or_create_tensor("b", [n])
    if bias_init:
        g.initializers["b"] = (rng.standard_normal(n) * 0.02).astype(np.float32)
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
    return g, w


def test_operator_fusion_pass_bias_and_activation():
    g, _ = _linear_graph(4, 32, 16, R.OperatorType_Gelu)
    assert R.OperatorFusionPass(1).run(g) == 1
    assert len(g.nodes) == 1
    nd = g.nodes[0]
    assert nd.op_type == R.OperatorType_FusedLinear
    assert nd.inputs == ["x", "W", "b"] and nd.outputs == ["y"]
    assert nd.activation == R.ActivationFunction_GELU
    assert R.OperatorFusionPass(1).run(g) == 0  # nothing left to fuse


def test_operator_fusion_pass_bias_must_be_initializer():
    g, _ = _linear_graph(4, 32, 16, bias_init=False)
    assert R.OperatorFusionPass(1).run(g) == 0  # session.tkv:3718: only an initializer bias fuses
    assert [n.op_type for n in g.nodes] == [R.OperatorType_MatMul, R.OperatorType_Add]


def test_operator_fusion_pass_matmul_then_relu_and_conv():
    g = R.ExecutionGraph()
    a = R.new_node("mm", R.OperatorType_MatMul)
    a.inputs, a.outputs = ["x", "W"], ["t"]
    r = R.new_node("r", R.OperatorType_Relu)
    r.inputs, r.outputs = ["t"], ["y"]
    c = R.new_node("c", R.OperatorType_Conv2D)
    c.inputs, c.outputs = ["y", "K"], ["u"]
    r2 = R.new_node("r2", R.OperatorType_Relu)
    r2.inputs, r2.outputs = ["u"], ["z"]
    g.nodes = [a, r, c, r2]
    assert R.OperatorFusionPass().run(g) == 1
    assert [(n.op_type, n.outputs) for n in g.nodes] == [(R.OperatorType_FusedLinear, ["y"]),
                                                         (R.OperatorType_FusedConv2D, ["z"])]
    assert g.nodes[0].activation == R.ActivationFunction_ReLU


def _artefact_for(name, n, k, act, seed=0, per_channel=True):
    rng = np.random.default_rng(seed)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    sw = (rng.random(n) * 1e-3 + 1e-4).astype(np.float32)
    b = (rng.standard_normal(n) * 0.02).astype(np.float32)
    if per_channel:
        return ptq.QuantLinear(name, w, scales_w=sw, bias=b, scale_a=0.031, act=act)
    return ptq.QuantLinear(name, w, scale_b=float(sw[0]), bias=b, scale_a=0.031, act=act)


def test_ptq_rewrite_from_artefact_structure():
    m, k, n = 8, 64, 48
    g, _ = _linear_graph(m, k, n, R.OperatorType_Gelu)
    R.OperatorFusionPass().run(g)
    q = _artefact_for("fc", n, k, R.ActivationFunction_GELU)
    p = R.PtqRewritePass(artefact=[q])
    assert p.run(g) == 1
    ops = [(nd.op_type, nd.inputs, nd.outputs) for nd in g.nodes]
    assert ops == [(R.OperatorType_Custom, ["x"], ["fc.x_q"]),
                   (R.OperatorType_QuantizedGemm, ["fc.x_q", "fc.w_q", "fc.bias"], ["fc.pre_act"]),
                   (R.OperatorType_Gelu, ["fc.pre_act"], ["y"])]
    quant, gemm = g.nodes[0], g.nodes[1]
    assert quant.custom == R.CUSTOM_QUANTIZE_INT8 and quant.scale_a == q.scale_a
    assert gemm.scale_a == q.scale_a and np.array_equal(np.float32(gemm.scales_w), q.scales_w)
    assert g.tensors["fc.x_q"].dtype == R.TensorDataType_Int8 and g.tensors["fc.x_q"].shape == [m, k]
    assert g.tensors["fc.w_q"].shape == [n, k]
    assert np.array_equal(g.initializers_int8["fc.w_q"], q.w)
    # the f32 weight is read by no node any more: gone from the arena
    assert "W" not in g.initializers and "W" not in g.tensors
    assert p.linears == [q]


def test_ptq_rewrite_export_round_trip(tmp_path):
    m, k, n = 2, 32, 16
    g, _ = _linear_graph(m, k, n)
    R.OperatorFusionPass().run(g)
    q = _artefact_for("fc", n, k, R.ActivationFunction_None, per_channel=False)
    R.PtqRewritePass(artefact=[q]).run(g)
    path = str(tmp_path / "g.tvqptq")
    assert R.export_ptq(g, path, {"graph": "lin"}) == 1
    back, meta = ptq.load(path)
    assert meta == {"graph": "lin"}
    assert back == [q]
    # and into a fresh copy of the graph from the file path
    g2, _ = _linear_graph(m, k, n)
    R.OperatorFusionPass().run(g2)
    assert R.PtqRewritePass(artefact=path).run(g2) == 1
    assert [nd.op_type for nd in g2.nodes] == [R.OperatorType_Custom, R.OperatorType_QuantizedGemm]
    assert g2.nodes[1].scales_w == [] and g2.nodes[1].scale_b == q.scale_b


def test_ptq_rewrite_leaves_linears_without_a_scale():
    g, _ = _linear_graph(4, 32, 16)
    R.OperatorFusionPass().run(g)
    assert R.PtqRewritePass().run(g) == 0
    assert [nd.op_type for nd in g.nodes] == [R.OperatorType_FusedLinear]
    assert "W" in g.initializers


def test_ptq_rewrite_skips_rank3_inputs():
    # QuantizedGemm's _m() takes shape[0] only (session.tkv:3029-3035): a
    # [2, 4, k] input would not be the linear's m = 8 rows
    g, _ = _linear_graph(8, 32, 16, x_shape=[2, 4, 32])
    R.OperatorFusionPass().run(g)
    assert R.PtqRewritePass(artefact=[_artefact_for("fc", 16, 32, 0)]).run(g) == 0


def test_ptq_rewrite_artefact_mismatch_raises():
    g, _ = _linear_graph(4, 32, 16)
    R.OperatorFusionPass().run(g)
    with pytest.raises(ValueError):
        R.PtqRewritePass(artefact=[_artefact_for("fc", 16, 64, 0)]).run(g)
    g, _ = _linear_graph(4, 32, 16, R.OperatorType_Relu)
    R.OperatorFusionPass().run(g)
    with pytest.raises(ValueError):  # the artefact was made for a linear without activation
        R.PtqRewritePass(artefact=[_artefact_for("fc", 16, 32, 0)]).run(g)


def test_ptq_rewrite_square_weight_is_n_by_k():
    # _exec_linear (session.tkv:756-761) tests shape[1] == k first: a square
    # weight is [N, K] whatever the graph meant
    g, _ = _linear_graph(4, 32, 32)
    R.OperatorFusionPass().run(g)
    assert R._linear_dims(g, g.nodes[0]) == (4, 32, 32, 1)


def test_ptq_rewrite_transposed_weight_dims():
    g, _ = _linear_graph(4, 32, 16, trans_b=True)  # W stored [n, k]
    R.OperatorFusionPass().run(g)
    assert R._linear_dims(g, g.nodes[0]) == (4, 16, 32, 1)
    g, _ = _linear_graph(4, 32, 16)
    R.OperatorFusionPass().run(g)
    assert R._linear_dims(g, g.nodes[0]) == (4, 16, 32, 0)
