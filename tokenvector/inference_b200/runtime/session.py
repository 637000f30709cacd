"""Mirror of tv/runtime/session.tkv for graphs of QuantizedGemm nodes.

Same names, constants and call shapes as the reference (ExecutionGraph,
ExecutionNode, InferenceSession.run / run_single, named_tensor /
named_qdata / named_idata, session_from_graph), executed on the B200: the
arena is one device allocation, initializers (f32 and int8) are uploaded once
at session construction (initialize_weights, session.tkv:3336-3350), and a
QuantizedGemm node runs the tcgen05 GEMM of libtvq with the node's scale_a and
scales_w (or scale_b) -- per-channel iff len(scales_w) > 0, the activation
field ignored, exactly as the reference's branch (session.tkv:678-697).

Also executable: the ONNX QDQ family (QuantizeLinear, DequantizeLinear,
QLinearMatMul, MatMulInteger, DynamicQuantizeLinear, session.tkv:1896-2071,
2789-2905), the QdqFoldPass graph pass (:3774-3804), and the PTQ rewrite
(PtqRewritePass): FusedLinear / MatMul over an f32 weight initializer becomes
a Custom QuantizeInt8Symmetric node (engine.tkv:216-226) feeding a
QuantizedGemm, its activation a Relu / Gelu node that the executor fuses
into the GEMM's epilogue.  Other operator types belong to the reference's
fp32 runtime and raise NotImplementedError.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .. import _native as N

# ---- enums, tv/runtime/session.tkv:274-294, 361-366, 372-444
TensorDataType_Undefined = 0
TensorDataType_Float = 1
TensorDataType_Uint8 = 2
TensorDataType_Int8 = 3
TensorDataType_Uint16 = 4
TensorDataType_Int16 = 5
TensorDataType_Int32 = 6
TensorDataType_Int64 = 7
TensorDataType_String = 8
TensorDataType_Bool = 9
TensorDataType_Float16 = 10
TensorDataType_Double = 11
TensorDataType_BFloat16 = 16
TensorDataType_Float8E4M3FN = 17
TensorDataType_Float8E5M2 = 19

ActivationFunction_None = 0
ActivationFunction_ReLU = 1
ActivationFunction_GELU = 2
ActivationFunction_SiLU = 3
ActivationFunction_Sigmoid = 4
ActivationFunction_Tanh = 5

OperatorType_Custom = 0
OperatorType_MatMul = 1
OperatorType_FusedLinear = 2
OperatorType_Conv2D = 3
OperatorType_FusedConv2D = 4
OperatorType_LayerNorm = 6
OperatorType_Attention = 7
OperatorType_Relu = 8
OperatorType_Gelu = 9
OperatorType_Silu = 10
OperatorType_Sigmoid = 11
OperatorType_Tanh = 12
OperatorType_Add = 13
OperatorType_QuantizedGemm = 21
OperatorType_Identity = 22
OperatorType_QuantizeLinear = 63
OperatorType_DequantizeLinear = 64
OperatorType_QLinearMatMul = 65
OperatorType_MatMulInteger = 78
OperatorType_DynamicQuantizeLinear = 79

# Custom operator of the PTQ rewrite: y int8 = quantize_int8_symmetric (x f32,
# node.scale_a).  ONNX QuantizeLinear is not the same function (x / s, clamp
# to [-128, 127], session.tkv:1917-1922; the reference's PTQ quantizes by
# x * fl32(1/s), clamp to [-127, 127]).
CUSTOM_QUANTIZE_INT8 = "QuantizeInt8Symmetric"

# the activation of a FusedLinear as its own operator (OperatorFusionPass,
# session.tkv:3733-3753, read backwards)
_ACT_OP = {ActivationFunction_ReLU: OperatorType_Relu, ActivationFunction_GELU: OperatorType_Gelu,
           ActivationFunction_SiLU: OperatorType_Silu, ActivationFunction_Sigmoid: OperatorType_Sigmoid,
           ActivationFunction_Tanh: OperatorType_Tanh}
# unary operators the QuantizedGemm epilogue evaluates as apply_activation
# (tv/optimization/kernels.tkv:14-38) does
_EPILOGUE_ACT = {OperatorType_Relu: N.ACT_RELU, OperatorType_Gelu: N.ACT_GELU_TANH}

QDQ_OPS = (OperatorType_QuantizeLinear, OperatorType_DequantizeLinear, OperatorType_QLinearMatMul,
           OperatorType_MatMulInteger, OperatorType_DynamicQuantizeLinear)


def calc_element_count(shape) -> int:
    """session.tkv:323-334"""
    if shape is None or len(shape) == 0:
        return 1
    total = 1
    for d in shape:
        total *= d if d > 0 else 1
    return total


def dtype_size(dtype: int) -> int:
    """session.tkv:336-350"""
    if dtype in (TensorDataType_Float, TensorDataType_Int32):
        return 4
    if dtype in (TensorDataType_Float16, TensorDataType_BFloat16):
        return 2
    if dtype in (TensorDataType_Int8, TensorDataType_Uint8, TensorDataType_Float8E4M3FN, TensorDataType_Float8E5M2):
        return 1
    if dtype in (TensorDataType_Int64, TensorDataType_Double):
        return 8
    return 4


class TensorDesc:
    """session.tkv:296-321"""

    def __init__(self, name: str, shape, dtype: int = TensorDataType_Float):
        self.name = name
        self.shape = list(shape)
        self.dtype = dtype
        self.element_count = calc_element_count(self.shape)
        self.byte_size = self.element_count * dtype_size(dtype)
        self.offset = -1
        self.is_input = 0
        self.is_output = 0
        self.is_initializer = 0


def make_tensor_desc(name: str, shape, dtype: int) -> TensorDesc:
    return TensorDesc(name, shape, dtype)


class ExecutionNode:
    """session.tkv:446-572 (the fields the PTQ path reads)."""

    def __init__(self, name: str, op: int):
        self.id = -1
        self.name = name
        self.op_type = op
        self.inputs: list = []
        self.outputs: list = []
        self.input_descs: list = []
        self.output_descs: list = []
        self.activation = ActivationFunction_None
        self.scale_a = 1.0
        self.scale_b = 1.0
        self.scale_y = 1.0
        self.zp_a = 0
        self.zp_b = 0
        self.zp_y = 0
        self.scales_w: list = []
        self.qlinear_axis = 1  # session.tkv:550
        self.custom = ""  # OperatorType_Custom: which custom operator

    # session.tkv:3029-3051
    def _m(self) -> int:
        a = self.input_descs[0]
        return a.shape[0] if len(a.shape) > 1 else 1

    def _k_gemm(self) -> int:
        a = self.input_descs[0]
        return a.shape[1] if len(a.shape) > 1 else a.element_count

    def _n_gemm(self) -> int:
        b = self.input_descs[1]
        return b.shape[0] if len(b.shape) > 1 else b.element_count


def new_node(name: str, op: int) -> ExecutionNode:
    """session.tkv:3130-3134"""
    return ExecutionNode(name, op)


class ExecutionGraph:
    """session.tkv:3141-3350"""

    def __init__(self, name: str = "TokenVectorGraph"):
        self.name = name
        self.nodes: list = []
        self.tensors: dict = {}
        self.inputs: list = []
        self.outputs: list = []
        self.initializers: dict = {}
        self.initializers_int8: dict = {}
        self.total_arena_bytes = 0

    def get_or_create_tensor(self, name: str, shape, dtype: int = TensorDataType_Float) -> TensorDesc:
        if name in self.tensors:
            t = self.tensors[name]
            if len(shape) > 0 and len(t.shape) == 0:
                t.shape = list(shape)
                t.element_count = calc_element_count(shape)
                t.byte_size = t.element_count * dtype_size(dtype)
            return t
        t = make_tensor_desc(name, shape, dtype)
        self.tensors[name] = t
        return t

    def analyze_liveness_and_allocate_offsets(self) -> int:
        """Device arena layout.  Every tensor gets its own 256-byte aligned
        slot (the arena lives in HBM, so the reference's greedy scratch reuse,
        session.tkv:3180-3326, buys nothing worth an aliasing hazard)."""
        off = 0
        for t in self.tensors.values():
            t.offset = off
            off += (max(t.byte_size, 1) + 255) // 256 * 256
        self.total_arena_bytes = off
        return 0


class QdqFoldPass:
    """session.tkv:3774-3804: a QuantizeLinear whose only output feeds the
    next node, a DequantizeLinear with one output, is removed together with
    it; readers of the DequantizeLinear output read the QuantizeLinear input
    instead (graph outputs too)."""

    def __init__(self, verbose: int = 1):
        self.verbose = verbose

    def name(self) -> str:
        return "QdqFoldPass"

    def run(self, graph: "ExecutionGraph") -> int:
        modified = 0
        i = 0
        while i < len(graph.nodes):
            node = graph.nodes[i]
            if node.op_type == OperatorType_QuantizeLinear and len(node.outputs) == 1 and i + 1 < len(graph.nodes):
                nxt = graph.nodes[i + 1]
                if (nxt.op_type == OperatorType_DequantizeLinear and len(nxt.inputs) > 0
                        and nxt.inputs[0] == node.outputs[0] and len(nxt.outputs) == 1):
                    orig, dead = node.inputs[0], nxt.outputs[0]
                    for nd in graph.nodes:
                        nd.inputs = [orig if x == dead else x for x in nd.inputs]
                    graph.outputs = [orig if x == dead else x for x in graph.outputs]
                    graph.nodes.pop(i + 1)
                    graph.nodes.pop(i)
                    modified = 1
                    continue
            i += 1
        return modified


class OperatorFusionPass:
    """session.tkv:3698-3771, the three rewrites in the reference's order:
    (1) MatMul then an Add of its output and a bias initializer -> one
    FusedLinear with the bias as third input; (2) FusedLinear / MatMul then a
    Relu / Gelu / Silu / Sigmoid / Tanh of its output -> the activation moves
    into the linear; (3) Conv2D then Relu -> FusedConv2D.  Each rewrite looks
    at adjacent node pairs only and takes over the second node's output."""

    _UNARY = {OperatorType_Relu: ActivationFunction_ReLU, OperatorType_Gelu: ActivationFunction_GELU,
              OperatorType_Silu: ActivationFunction_SiLU, OperatorType_Sigmoid: ActivationFunction_Sigmoid,
              OperatorType_Tanh: ActivationFunction_Tanh}

    def __init__(self, verbose: int = 1):
        self.verbose = verbose

    def name(self) -> str:
        return "OperatorFusionPass"

    @staticmethod
    def _sweep(graph: "ExecutionGraph", merge) -> int:
        modified = 0
        i = 0
        while i < len(graph.nodes) - 1:
            if merge(graph, graph.nodes[i], graph.nodes[i + 1]):
                graph.nodes.pop(i + 1)  # the pair may fuse again with the next node
                modified = 1
            else:
                i += 1
        return modified

    @staticmethod
    def _bias(graph, a, b) -> bool:
        if a.op_type != OperatorType_MatMul or b.op_type != OperatorType_Add or not a.outputs or len(b.inputs) < 2:
            return False
        y = a.outputs[0]
        if y not in b.inputs[:2]:
            return False
        bias = b.inputs[1] if b.inputs[0] == y else b.inputs[0]
        if bias not in graph.initializers:
            return False
        a.op_type = OperatorType_FusedLinear
        a.inputs.append(bias)
        a.outputs[0] = b.outputs[0]
        return True

    @classmethod
    def _act(cls, graph, a, b) -> bool:
        if a.op_type not in (OperatorType_FusedLinear, OperatorType_MatMul) or b.op_type not in cls._UNARY:
            return False
        if not a.outputs or not b.inputs or a.outputs[0] != b.inputs[0]:
            return False
        a.op_type = OperatorType_FusedLinear
        a.activation = cls._UNARY[b.op_type]
        a.outputs[0] = b.outputs[0]
        return True

    @staticmethod
    def _conv(graph, a, b) -> bool:
        if a.op_type != OperatorType_Conv2D or b.op_type != OperatorType_Relu:
            return False
        if not a.outputs or not b.inputs or a.outputs[0] != b.inputs[0]:
            return False
        a.op_type = OperatorType_FusedConv2D
        a.outputs[0] = b.outputs[0]
        return True

    def run(self, graph: "ExecutionGraph") -> int:
        m1 = self._sweep(graph, self._bias)
        m2 = self._sweep(graph, self._act)
        m3 = self._sweep(graph, self._conv)
        return 1 if (m1 or m2 or m3) else 0


def _linear_dims(graph: "ExecutionGraph", node: ExecutionNode):
    """(m, n, k, trans_b) of a MatMul / FusedLinear the way _exec_linear
    reads them (session.tkv:736-766): k = last dim of A, m = the product of
    the others; a 2-D B is [N, K] when its second dim is K, else [K, N]."""
    a = graph.tensors[node.inputs[0]]
    b = graph.tensors[node.inputs[1]]
    if len(a.shape) > 1:
        k = a.shape[-1]
        m = int(np.prod(a.shape[:-1]))
    else:
        k, m = a.element_count, 1
    if len(b.shape) != 2:
        return None
    if b.shape[1] == k:
        return m, b.shape[0], k, 1
    if b.shape[0] == k:
        return m, b.shape[1], k, 0
    return None


class PtqRewritePass:
    """Post-training quantization of the graph's linears: every MatMul /
    FusedLinear whose weight is an f32 initializer and whose input has an
    activation scale becomes

        x --[Custom QuantizeInt8Symmetric, scale_a]--> x_q (int8)
        x_q, W_q, bias --[QuantizedGemm, scale_a, scales_w]--> y (f32)
        (+ y_pre --[Relu | Gelu | ...]--> y for a fused activation)

    the reference's PTQ recipe (engine.tkv): W per output channel
    (calibrate_per_channel_minmax + quantize_int8_per_channel on W as [N, K],
    :202-250), x symmetric per tensor (calibrate_minmax, :13-36, over the
    given batches) and a QuantizedGemm node (session.tkv:678-697), which
    ignores node.activation -- the activation stays a node of its own.

    Scale sources, first match wins: `artefact` (a TVQPTQ1 file, or the list
    that ptq.load returns; entries by node name, nothing recalibrated),
    `act_scales` {input tensor name: scale_a}, `calibration` {input tensor
    name: [f32 batches]}.  A linear with none keeps its fp32 form."""

    def __init__(self, act_scales: dict | None = None, calibration: dict | None = None, artefact=None,
                 verbose: int = 1):
        self.act_scales = dict(act_scales or {})
        self.calibration = dict(calibration or {})
        if isinstance(artefact, str):
            from ..ptq import load
            artefact = load(artefact)[0]
        self.artefact = {q.name: q for q in (artefact or [])}
        self.verbose = verbose
        self.linears: list = []  # the QuantLinear of every rewritten node, in graph order

    def name(self) -> str:
        return "PtqRewritePass"

    def _quant_linear(self, graph: "ExecutionGraph", node: ExecutionNode):
        from ..ptq import QuantLinear
        if node.op_type not in (OperatorType_MatMul, OperatorType_FusedLinear) or len(node.inputs) < 2:
            return None
        if node.inputs[0] not in graph.tensors or node.inputs[1] not in graph.tensors:
            return None
        if len(graph.tensors[node.inputs[0]].shape) > 2:
            return None  # QuantizedGemm's _m() reads shape[0] only (session.tkv:3029-3035)
        dims = _linear_dims(graph, node)
        if dims is None:
            return None
        m, n, k, trans_b = dims
        bias_name = node.inputs[2] if len(node.inputs) > 2 else None
        if node.name in self.artefact:
            q = self.artefact[node.name]
            if (q.n, q.k) != (n, k):
                raise ValueError("artefact linear %r is [%d, %d], the graph's [%d, %d]" % (node.name, q.n, q.k, n, k))
            if q.act != node.activation:
                raise ValueError("artefact linear %r has activation %d, the graph's node %d"
                                 % (node.name, q.act, node.activation))
            return q
        wname = node.inputs[1]
        if wname not in graph.initializers:
            return None
        x = node.inputs[0]
        if x in self.act_scales:
            scale_a = float(self.act_scales[x])
        elif x in self.calibration:
            from ..quantization.engine import calibrate_minmax_batches
            scale_a = calibrate_minmax_batches(self.calibration[x], 1).scale
        else:
            return None
        from ..quantization.engine import calibrate_per_channel_minmax, quantize_int8_per_channel
        w = np.asarray(graph.initializers[wname], np.float32).ravel()[:n * k]
        w_nk = np.ascontiguousarray(w.reshape(n, k) if trans_b else w.reshape(k, n).T)
        scales = np.array([p.scale for p in calibrate_per_channel_minmax(w_nk, n, k, 1)], np.float32)
        wq = np.empty((n, k), np.int8)
        quantize_int8_per_channel(w_nk, wq, n, k, scales)
        bias = None
        if bias_name is not None and bias_name in graph.initializers:
            bias = np.asarray(graph.initializers[bias_name], np.float32).ravel()[:n]
        return QuantLinear(node.name, wq, scales_w=scales, bias=bias, scale_a=scale_a, act=node.activation)

    def _rewrite(self, graph: "ExecutionGraph", node: ExecutionNode, q) -> list:
        x = node.inputs[0]
        xd = graph.tensors[x]
        xq = node.name + ".x_q"
        graph.get_or_create_tensor(xq, xd.shape, TensorDataType_Int8)
        wq = node.name + ".w_q"
        graph.get_or_create_tensor(wq, [q.n, q.k], TensorDataType_Int8)
        graph.initializers_int8[wq] = q.w
        quant = new_node(node.name + ".quantize", OperatorType_Custom)
        quant.custom = CUSTOM_QUANTIZE_INT8
        quant.inputs, quant.outputs = [x], [xq]
        quant.scale_a = q.scale_a
        gemm = new_node(node.name, OperatorType_QuantizedGemm)
        gemm.inputs = [xq, wq]
        bias_in = node.inputs[2] if len(node.inputs) > 2 else None
        if q.bias is not None:
            # the QuantLinear's bias, bit for bit (an artefact reproduces the
            # session that wrote it): the graph's own initializer where equal
            held = graph.initializers.get(bias_in) if bias_in is not None else None
            same = held is not None and np.array_equal(
                np.asarray(held, np.float32).ravel()[:q.n].view(np.uint32), q.bias[:q.n].view(np.uint32))
            if not same:
                bias_in = node.name + ".bias"
                graph.get_or_create_tensor(bias_in, [q.n], TensorDataType_Float)
                graph.initializers[bias_in] = q.bias[:q.n]
        if bias_in is not None:
            gemm.inputs.append(bias_in)
        gemm.scale_a = q.scale_a
        if q.scales_w is not None:
            gemm.scales_w = [float(v) for v in q.scales_w]
        else:
            gemm.scale_b = q.scale_b
        out = [quant, gemm]
        if q.act == ActivationFunction_None:
            gemm.outputs = list(node.outputs)
        else:
            if q.act not in _ACT_OP:
                raise ValueError("unknown activation %d" % q.act)
            pre = node.name + ".pre_act"
            yd = graph.tensors[node.outputs[0]]
            graph.get_or_create_tensor(pre, yd.shape, TensorDataType_Float)
            gemm.outputs = [pre]
            act = new_node(node.name + ".act", _ACT_OP[q.act])
            act.inputs, act.outputs = [pre], list(node.outputs)
            out.append(act)
        return out

    def run(self, graph: "ExecutionGraph") -> int:
        modified = 0
        i = 0
        while i < len(graph.nodes):
            node = graph.nodes[i]
            q = self._quant_linear(graph, node)
            if q is None:
                i += 1
                continue
            new = self._rewrite(graph, node, q)
            graph.nodes[i:i + 1] = new
            self.linears.append(q)
            i += len(new)
            modified = 1
        # f32 weights that no node reads any more
        read = {t for nd in graph.nodes for t in nd.inputs}
        for name in [t for t in list(graph.initializers) if t not in read and t not in graph.outputs]:
            if name in graph.tensors and graph.tensors[name].dtype == TensorDataType_Float:
                del graph.initializers[name]
                del graph.tensors[name]
        return modified


def export_ptq(graph: "ExecutionGraph", path: str, meta: dict | None = None) -> int:
    """Write the graph's QuantizedGemm nodes as a TVQPTQ1 artefact (int8
    weights, scales_w / scale_b, bias, scale_a, and the activation of a
    directly following Relu / Gelu / ... node): the input of
    PtqRewritePass(artefact=path).  Returns the number of linears written."""
    from ..ptq import QuantLinear, save
    act_of = {v: k for k, v in _ACT_OP.items()}
    out = []
    for i, nd in enumerate(graph.nodes):
        if nd.op_type != OperatorType_QuantizedGemm:
            continue
        wname = nd.inputs[1]
        if wname not in graph.initializers_int8:
            raise ValueError("QuantizedGemm %r: weight %r is not an int8 initializer" % (nd.name, wname))
        wd = graph.tensors[wname]
        n, k = (wd.shape[0], wd.shape[1]) if len(wd.shape) == 2 else (1, wd.element_count)
        w = np.asarray(graph.initializers_int8[wname]).ravel().astype(np.int64).astype(np.int8).reshape(n, k)
        bias = None
        if len(nd.inputs) > 2 and nd.inputs[2] in graph.initializers:
            bias = np.asarray(graph.initializers[nd.inputs[2]], np.float32).ravel()[:n]
        act = ActivationFunction_None
        if i + 1 < len(graph.nodes):
            nx = graph.nodes[i + 1]
            if nx.op_type in act_of and nx.inputs[:1] == nd.outputs[:1]:
                act = act_of[nx.op_type]
        per_channel = len(nd.scales_w) > 0
        out.append(QuantLinear(nd.name, w, scales_w=np.asarray(nd.scales_w, np.float32) if per_channel else None,
                               bias=bias, scale_a=nd.scale_a, scale_b=None if per_channel else nd.scale_b, act=act))
    save(path, out, meta)
    return len(out)


class NamedTensor:
    """session.tkv:3376-3387"""

    def __init__(self, name: str, data=None, qdata=None, idata=None):
        self.name = name
        self.data = data if data is not None else []
        self.qdata = qdata if qdata is not None else []
        self.idata = idata if idata is not None else []


def named_tensor(name: str, data) -> NamedTensor:
    return NamedTensor(name, data=data)


def named_qdata(name: str, qdata) -> NamedTensor:
    return NamedTensor(name, qdata=qdata)


def named_idata(name: str, idata) -> NamedTensor:
    return NamedTensor(name, idata=idata)


class Disposed(Exception):
    pass


_TORCH_DT = None


def _torch_dtype(dt):
    import torch
    return {TensorDataType_Float: torch.float32, TensorDataType_Int8: torch.int8, TensorDataType_Uint8: torch.uint8,
            TensorDataType_Int32: torch.int32, TensorDataType_Int64: torch.int64,
            TensorDataType_Float8E4M3FN: torch.uint8}[dt]


class InferenceSession:
    """session.tkv:3389-3503 on the GPU."""

    def __init__(self, graph: ExecutionGraph, apply_optimizations: int = 1, device: int = 0, ptq=None):
        import torch
        self.graph = graph
        self.device = torch.device("cuda", device)
        self._disposed = 0
        if apply_optimizations:
            # session.tkv:3388-3396; constant folding and dead-code
            # elimination act on the fp32 operators, outside this path
            QdqFoldPass(1).run(graph)
            OperatorFusionPass(1).run(graph)
        if ptq is not None:  # a PtqRewritePass: the graph's linears to INT8
            ptq.run(graph)
        # resolve node tensor descriptors (the reference binds them at graph build)
        for node in graph.nodes:
            node.input_descs = [graph.tensors[n] for n in node.inputs]
            node.output_descs = [graph.tensors[n] for n in node.outputs]
        graph.analyze_liveness_and_allocate_offsets()
        self.arena = torch.zeros(max(graph.total_arena_bytes, 256), dtype=torch.uint8, device=self.device)
        self._initialize_weights()
        self._fused = self._plan_epilogue_fusion()
        self._prep = [self._prepare(i, n) for i, n in enumerate(graph.nodes)]

    def _plan_epilogue_fusion(self) -> dict:
        """{index of a QuantizedGemm: index of the Relu / Gelu node it absorbs}
        where the unary node reads the GEMM's output and nothing else does
        (the intermediate is then never materialised)."""
        g = self.graph
        readers: dict = {}
        for nd in g.nodes:
            for t in nd.inputs:
                readers[t] = readers.get(t, 0) + 1
        fused = {}
        for i in range(len(g.nodes) - 1):
            a, b = g.nodes[i], g.nodes[i + 1]
            if (a.op_type == OperatorType_QuantizedGemm and b.op_type in _EPILOGUE_ACT and b.inputs[:1] == a.outputs[:1]
                    and readers.get(a.outputs[0], 0) == 1 and a.outputs[0] not in g.outputs):
                fused[i] = i + 1
        return fused

    # arena views
    def _view(self, desc: TensorDesc):
        import torch
        dt = _torch_dtype(desc.dtype)
        nbytes = desc.element_count * dtype_size(desc.dtype)
        return self.arena[desc.offset:desc.offset + nbytes].view(dt)

    def _initialize_weights(self):
        import torch
        g = self.graph
        for nm, vals in g.initializers.items():
            if nm in g.tensors:
                self._view(g.tensors[nm]).copy_(torch.as_tensor(np.asarray(vals, np.float32).ravel()))
        for nm, vals in g.initializers_int8.items():
            if nm in g.tensors:
                v = np.asarray(vals).ravel().astype(np.int64).astype(np.int8)
                self._view(g.tensors[nm]).copy_(torch.as_tensor(v).view(_torch_dtype(g.tensors[nm].dtype)))

    def _scalar(self, desc: TensorDesc) -> float:
        """_span0 (session.tkv:25-27): element 0 of a float span."""
        nm = desc.name
        if nm in self.graph.initializers:
            return float(np.asarray(self.graph.initializers[nm], np.float32).ravel()[0])
        return float(self._view(desc)[:1].cpu().numpy()[0])

    def _axis_split(self, desc: TensorDesc, nsc: int, axis: int):
        """(outer, dim, inner) at the node's qlinear_axis (session.tkv:1926-1940)."""
        if nsc == 1:
            return 1, desc.element_count, 1
        rank = len(desc.shape)
        ax = axis if axis >= 0 else axis + rank
        outer = int(np.prod(desc.shape[:ax])) if ax > 0 else 1
        inner = int(np.prod(desc.shape[ax + 1:])) if ax + 1 < rank else 1
        return outer, int(desc.shape[ax]), inner

    def _prepare(self, idx: int, node: ExecutionNode):
        import torch
        if node.op_type == OperatorType_Identity:
            return None
        if node.op_type in QDQ_OPS:
            return None
        if idx in self._fused.values():
            return "fused"  # evaluated by the preceding QuantizedGemm's epilogue
        if node.op_type == OperatorType_Custom:
            if node.custom != CUSTOM_QUANTIZE_INT8:
                raise NotImplementedError("custom operator %r" % node.custom)
            if node.input_descs[0].dtype != TensorDataType_Float or node.output_descs[0].dtype != TensorDataType_Int8:
                raise ValueError("QuantizeInt8Symmetric: f32 input, int8 output")
            return dict(sa=torch.tensor([node.scale_a], dtype=torch.float32, device=self.device))
        if node.op_type != OperatorType_QuantizedGemm:
            raise NotImplementedError("operator %d is outside the PTQ path this runtime executes" % node.op_type)
        m, n, k = node._m(), node._n_gemm(), node._k_gemm()
        per_channel = len(node.scales_w) > 0
        if per_channel and len(node.scales_w) < n:
            raise ValueError("scales_w smaller than N")  # matmul.tkv:18-19
        sa = torch.tensor([node.scale_a], dtype=torch.float32, device=self.device)
        sw = torch.tensor(list(node.scales_w) if per_channel else [node.scale_b], dtype=torch.float32,
                          device=self.device)
        kp = (k + 15) // 16 * 16
        pad = None
        if kp != k:  # TMA row pitch: zero-padded copies of A and W (exact for the dot products)
            pad = (torch.zeros((m, kp), dtype=torch.int8, device=self.device),
                   torch.zeros((n, kp), dtype=torch.int8, device=self.device))
        act, out = N.ACT_NONE, node.output_descs[0]
        if idx in self._fused:
            un = self.graph.nodes[self._fused[idx]]
            act, out = _EPILOGUE_ACT[un.op_type], un.output_descs[0]
        return dict(m=m, n=n, k=k, kp=kp, sa=sa, sw=sw, per_channel=per_channel, pad=pad, act=act, out=out)

    def _exec_qdq(self, node: ExecutionNode, stream):
        """The QDQ operator family, session.tkv:1896-2071 and 2789-2905."""
        ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
        ins, outs = node.input_descs, node.output_descs
        op = node.op_type
        if op in (OperatorType_QuantizeLinear, OperatorType_DequantizeLinear):
            x, sc, y = ins[0], ins[1], outs[0]
            zp = int(self._scalar(ins[2])) if len(ins) > 2 else 0
            outer, dim, inner = self._axis_split(x, sc.element_count, node.qlinear_axis)
            fn = "tvq_dev_quantize_linear" if op == OperatorType_QuantizeLinear else "tvq_dev_dequantize_linear"
            N.call(fn, ptr(self._view(x)), ptr(self._view(y)), outer, dim, inner, ptr(self._view(sc)),
                   sc.element_count, zp, stream)
        elif op in (OperatorType_MatMulInteger, OperatorType_QLinearMatMul):
            ad = ins[0]
            bd = ins[1] if op == OperatorType_MatMulInteger else ins[3]
            m = ad.shape[0] if len(ad.shape) > 0 else 1
            if op == OperatorType_QLinearMatMul and len(ad.shape) <= 1:
                m = 1
            k = ad.shape[1] if len(ad.shape) > 1 else ad.element_count
            n = bd.shape[1] if len(bd.shape) > 1 else bd.element_count
            a, b, y = self._view(ad), self._view(bd), self._view(outs[0])
            if op == OperatorType_MatMulInteger:
                N.call("tvq_dev_matmul_integer", ptr(a), ptr(b), ptr(y), m, k, n, stream)
            else:
                sa, zpa = self._scalar(ins[1]), int(self._scalar(ins[2]))
                sw, zpw = self._scalar(ins[4]), int(self._scalar(ins[5]))
                sy, zpy = self._scalar(ins[6]), int(self._scalar(ins[7]))
                N.call("tvq_dev_qlinear_matmul", ptr(a), sa, zpa, ptr(b), sw, zpw, sy, zpy, ptr(y), m, k, n, stream)
        else:  # DynamicQuantizeLinear
            x = ins[0]
            N.call("tvq_dev_dynamic_quantize_linear", ptr(self._view(x)), x.element_count,
                   ptr(self._view(outs[0])), ptr(self._view(outs[1])), ptr(self._view(outs[2])), stream)

    def _exec(self, node: ExecutionNode, prep):
        import torch
        if prep == "fused":
            return
        if node.op_type == OperatorType_Identity:
            self._view(node.output_descs[0]).copy_(self._view(node.input_descs[0]))
            return
        if node.op_type == OperatorType_Custom:  # QuantizeInt8Symmetric
            x = self._view(node.input_descs[0])
            N.call("tvq_dev_quantize_int8", C.c_void_p(x.data_ptr()),
                   C.c_void_p(self._view(node.output_descs[0]).data_ptr()), x.numel(),
                   C.c_void_p(prep["sa"].data_ptr()),
                   C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
            return
        if node.op_type in QDQ_OPS:
            self._exec_qdq(node, C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
            return
        a = self._view(node.input_descs[0])
        w = self._view(node.input_descs[1])
        y = self._view(prep["out"])
        bias = self._view(node.input_descs[2]) if len(node.input_descs) > 2 else None
        m, n, k, kp = prep["m"], prep["n"], prep["k"], prep["kp"]
        if prep["pad"] is not None:
            pa, pw = prep["pad"]
            pa[:, :k].copy_(a.view(m, k))
            pw[:, :k].copy_(w.view(n, k))
            a, w = pa, pw
        stream = torch.cuda.current_stream(self.device).cuda_stream
        ptr = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
        N.call("tvq_dev_gemm", N.GEMM_I8, ptr(a), ptr(w), ptr(bias), None, ptr(y), None, m, n, kp,
               ptr(prep["sa"]), ptr(prep["sw"]), 1 if prep["per_channel"] else 0, prep["act"], None, None,
               C.c_void_p(stream))

    def run(self, inputs: list, outputs: list) -> int:
        """session.tkv:3403-3436"""
        import torch
        if self._disposed:
            raise Disposed("InferenceSession")
        g = self.graph
        for inp in inputs:
            if inp.name in g.tensors:
                desc = g.tensors[inp.name]
                if len(inp.qdata) > 0:
                    v = np.asarray(inp.qdata).ravel().astype(np.int64).astype(np.int8)
                    self._view(desc)[:v.size].copy_(torch.as_tensor(v).view(_torch_dtype(desc.dtype)))
                elif len(inp.idata) > 0:
                    v = np.asarray(inp.idata).ravel().astype(np.int32)
                    self._view(desc)[:v.size].copy_(torch.as_tensor(v))
                else:
                    v = np.asarray(inp.data, np.float32).ravel()
                    self._view(desc)[:v.size].copy_(torch.as_tensor(v))
        for node, prep in zip(g.nodes, self._prep):
            self._exec(node, prep)
        torch.cuda.synchronize(self.device)
        N.call("tvq_device_error", None)
        for out in outputs:
            if out.name in g.tensors:
                desc = g.tensors[out.name]
                host = self._view(desc).cpu().numpy()
                if isinstance(out.data, np.ndarray) and out.data.size and len(out.qdata) == 0 and len(out.idata) == 0:
                    out.data.ravel()[:] = host.ravel()[:out.data.size]
                elif isinstance(out.qdata, np.ndarray) and out.qdata.size:
                    out.qdata.ravel()[:] = host.ravel()[:out.qdata.size]
                elif isinstance(out.idata, np.ndarray) and out.idata.size:
                    out.idata.ravel()[:] = host.ravel()[:out.idata.size]
                else:
                    out.data = host.ravel().astype(np.float32)
        return 0

    def run_single(self, input, input_name: str = "", output_name: str = ""):
        """session.tkv:3438-3500: one f32 input, one f32 output."""
        g = self.graph
        iname = input_name or g.inputs[0]
        oname = output_name or g.outputs[0]
        out = NamedTensor(oname, data=np.empty(g.tensors[oname].element_count, np.float32))
        self.run([named_tensor(iname, input)], [out])
        return out.data

    def close(self):
        self._disposed = 1
        self.arena = None


def session_from_graph(graph: ExecutionGraph, apply_optimizations: int = 1, device: int = 0,
                       ptq=None) -> InferenceSession:
    """session.tkv:3626 (ptq: an optional PtqRewritePass run on the graph first)"""
    return InferenceSession(graph, apply_optimizations, device, ptq)
