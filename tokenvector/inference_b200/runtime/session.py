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
2789-2905) and the QdqFoldPass graph pass (:3774-3804).  Other operator types
belong to the reference's fp32 runtime and raise NotImplementedError.
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
OperatorType_LayerNorm = 6
OperatorType_Attention = 7
OperatorType_Gelu = 9
OperatorType_Add = 13
OperatorType_QuantizedGemm = 21
OperatorType_Identity = 22
OperatorType_QuantizeLinear = 63
OperatorType_DequantizeLinear = 64
OperatorType_QLinearMatMul = 65
OperatorType_MatMulInteger = 78
OperatorType_DynamicQuantizeLinear = 79

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

    def __init__(self, graph: ExecutionGraph, apply_optimizations: int = 1, device: int = 0):
        import torch
        self.graph = graph
        self.device = torch.device("cuda", device)
        self._disposed = 0
        if apply_optimizations:
            # session.tkv:3388-3396; constant folding, operator fusion and
            # dead-code elimination act on the fp32 operators, outside this path
            QdqFoldPass(1).run(graph)
        # resolve node tensor descriptors (the reference binds them at graph build)
        for node in graph.nodes:
            node.input_descs = [graph.tensors[n] for n in node.inputs]
            node.output_descs = [graph.tensors[n] for n in node.outputs]
        graph.analyze_liveness_and_allocate_offsets()
        self.arena = torch.zeros(max(graph.total_arena_bytes, 256), dtype=torch.uint8, device=self.device)
        self._initialize_weights()
        self._prep = [self._prepare(n) for n in graph.nodes]

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

    def _prepare(self, node: ExecutionNode):
        import torch
        if node.op_type == OperatorType_Identity:
            return None
        if node.op_type in QDQ_OPS:
            return None
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
        return dict(m=m, n=n, k=k, kp=kp, sa=sa, sw=sw, per_channel=per_channel, pad=pad)

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
        if node.op_type == OperatorType_Identity:
            self._view(node.output_descs[0]).copy_(self._view(node.input_descs[0]))
            return
        if node.op_type in QDQ_OPS:
            self._exec_qdq(node, C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
            return
        a = self._view(node.input_descs[0])
        w = self._view(node.input_descs[1])
        y = self._view(node.output_descs[0])
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
               ptr(prep["sa"]), ptr(prep["sw"]), 1 if prep["per_channel"] else 0, N.ACT_NONE, None, None,
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


def session_from_graph(graph: ExecutionGraph, apply_optimizations: int = 1, device: int = 0) -> InferenceSession:
    """session.tkv:3626"""
    return InferenceSession(graph, apply_optimizations, device)
