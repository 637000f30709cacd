"""GPT-2-shaped INT8 PTQ forward on the B200: model weights, batch layout and
the native session (tvq_session_* in include/tvq.h).

The model is the reference's tv/training/gpt2_ref.tkv (LayerNorm eps 1e-6,
HF Conv1D weights [in, out], QKV split Q|K|V with heads contiguous, causal
softmax, erf GELU, tied LM head) with its four linears per block replaced by
QuantizedGemm nodes (tv/runtime/session.tkv:678-697): per-output-channel
INT8 weights, per-tensor static INT8 activations calibrated by one forward.
Attention, LayerNorm, GELU and the LM head stay fp32.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _native as N


@dataclass
class GPT2Config:
    vocab: int = 50257
    d_model: int = 768
    n_heads: int = 12
    n_layers: int = 12
    d_ffn: int = 3072
    max_pos: int = 1024
    eps: float = 1e-6          # gpt2_ref.tkv:35

    @staticmethod
    def gpt2_124m() -> "GPT2Config":
        return GPT2Config()

    @staticmethod
    def gpt2_xl_shape() -> "GPT2Config":
        return GPT2Config(vocab=50257, d_model=1600, n_heads=25, n_layers=48, d_ffn=6400, max_pos=1024)


# ---------------------------------------------------------------- synthetic init
_LCG_A, _LCG_C, _LCG_M = 1103515245, 12345, 2147483648


def _lcg_states(seed: int, count: int) -> np.ndarray:
    """`count` successive states of the LCG of gpt2_ref.tkv:1977-1978,
    vectorised with the jump-ahead s[i+B] = A_B s[i] + C_B (mod 2^31)."""
    B = 4096
    first = np.empty(min(B, count), np.int64)
    s = seed % _LCG_M
    for i in range(first.size):
        s = (s * _LCG_A + _LCG_C) % _LCG_M
        first[i] = s
    if count <= B:
        return first
    a_b, c_b = 1, 0
    for _ in range(B):  # compose B steps: x -> a x + c
        a_b, c_b = (a_b * _LCG_A) % _LCG_M, (c_b * _LCG_A + _LCG_C) % _LCG_M
    out = np.empty(count, np.int64)
    out[:B] = first
    cur = first
    for o in range(B, count, B):
        cur = (cur * a_b + c_b) % _LCG_M
        n = min(B, count - o)
        out[o:o + n] = cur[:n]
    return out


def gi_noise(n: int, seed: int, mult: float = 0.02) -> np.ndarray:
    """_gi_noise, tv/training/gpt2_ref.tkv:1980-1991: Box-Muller on pairs of
    LCG draws, times `mult` (0.02 for weights; 1.0 gives N(0, 1))."""
    st = _lcg_states(seed, 2 * n)
    u1 = (st[0::2].astype(np.float64) + 0.5) / 2147483648.0
    u2 = st[1::2].astype(np.float64) / 2147483648.0
    return (np.sqrt(0.0 - 2.0 * np.log(u1)) * np.cos(6.283185307179586 * u2) * mult).astype(np.float32)


@dataclass
class GPT2Weights:
    """fp32 weights in the reference's layout (gpt2_init, gpt2_ref.tkv:1997-2026)."""
    cfg: GPT2Config
    wte: np.ndarray
    wpe: np.ndarray
    lnf_g: np.ndarray
    lnf_b: np.ndarray
    layers: list = field(default_factory=list)  # dicts: ln1_g ln1_b attn_w attn_b proj_w proj_b ln2_g ln2_b fc_w fc_b mp_w mp_b

    @staticmethod
    def random(cfg: GPT2Config, seed: int = 0) -> "GPT2Weights":
        d = cfg.d_model
        w = GPT2Weights(cfg, gi_noise(cfg.vocab * d, seed + 1).reshape(cfg.vocab, d),
                        gi_noise(cfg.max_pos * d, seed + 2).reshape(cfg.max_pos, d), np.ones(d, np.float32),
                        np.zeros(d, np.float32))
        w.layers = random_layers(cfg, seed)
        return w


def random_layers(cfg: GPT2Config, seed: int = 0) -> list:
    """The blocks of gpt2_init (gpt2_ref.tkv:1997-2026): N(0, 0.02) linears,
    zero biases, LayerNorm gamma 1 / beta 0; layer l draws from seeds
    seed + 10 + 100 l + (1..4)."""
    d, f = cfg.d_model, cfg.d_ffn
    ones = lambda n: np.ones(n, np.float32)  # noqa: E731
    zeros = lambda n: np.zeros(n, np.float32)  # noqa: E731
    out = []
    for li in range(cfg.n_layers):
        sd = seed + 10 + li * 100
        out.append(dict(
            ln1_g=ones(d), ln1_b=zeros(d),
            attn_w=gi_noise(d * 3 * d, sd + 1).reshape(d, 3 * d), attn_b=zeros(3 * d),
            proj_w=gi_noise(d * d, sd + 2).reshape(d, d), proj_b=zeros(d),
            ln2_g=ones(d), ln2_b=zeros(d),
            fc_w=gi_noise(d * f, sd + 3).reshape(d, f), fc_b=zeros(f),
            mp_w=gi_noise(f * d, sd + 4).reshape(f, d), mp_b=zeros(d)))
    return out


LINEARS = (("attn_w", "attn_b"), ("proj_w", "proj_b"), ("fc_w", "fc_b"), ("mp_w", "mp_b"))


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def segments_from_lengths(lengths) -> np.ndarray:
    seg = np.zeros(len(lengths) + 1, np.int64)
    seg[1:] = np.cumsum(np.asarray(lengths, np.int64))
    return seg


def _f32(a):
    return np.ascontiguousarray(a, np.float32)


class _Session:
    """One tvq session: the blocks' weights, batch layout and scales."""

    # names of the four linears of a block in PTQ artefacts (HF GPT-2 naming)
    LINEAR_NAMES = ("attn.c_attn", "attn.c_proj", "mlp.c_fc", "mlp.c_proj")

    def __init__(self, cfg: GPT2Config, layers: list, vocab: int, device: int, max_tokens: int, ptq_path=None):
        self.cfg = cfg
        self.device = device
        h = C.c_int64()
        N.call("tvq_session_create", device, vocab, cfg.d_model, cfg.n_heads, cfg.n_layers, cfg.d_ffn,
               cfg.max_pos, float(cfg.eps), max_tokens, C.byref(h))
        self.handle = h.value
        self.max_tokens = max_tokens
        self._bias = []
        for li, L in enumerate(layers):
            N.call("tvq_session_set_layernorm", self.handle, li, 0, _p(_f32(L["ln1_g"])), _p(_f32(L["ln1_b"])))
            N.call("tvq_session_set_layernorm", self.handle, li, 1, _p(_f32(L["ln2_g"])), _p(_f32(L["ln2_b"])))
            self._bias.append([_f32(L[bk]) for _, bk in LINEARS])
            if ptq_path is None:
                for which, (wk, bk) in enumerate(LINEARS):
                    N.call("tvq_session_set_linear_f32", self.handle, li, which, _p(_f32(L[wk])), _p(_f32(L[bk])), 0)
        self.seg = None
        self.logits_mode = 0
        if ptq_path is not None:
            self.load_ptq(ptq_path)

    # ---- PTQ artefacts (ptq.py): the calibrated INT8 linears, reloaded bit-exact
    def export_ptq(self, path: str, meta: dict | None = None) -> None:
        """Write every block's INT8 linears (weights [n, k], per-channel
        scales, bias) with their calibrated activation scales."""
        from . import ptq
        sc = self.act_scales()
        lins = []
        for li in range(self.cfg.n_layers):
            for which, nm in enumerate(self.LINEAR_NAMES):
                w, sw = self.linear_i8(li, which)
                lins.append(ptq.QuantLinear("h.%d.%s" % (li, nm), w, scales_w=sw, bias=self._bias[li][which],
                                            scale_a=float(sc[li, which]), act=N.ACT_GELU_ERF if which == 2 else 0))
        c = self.cfg
        m = {"model": "gpt2-blocks", "d_model": c.d_model, "n_heads": c.n_heads, "n_layers": c.n_layers,
             "d_ffn": c.d_ffn}
        m.update(meta or {})
        ptq.save(path, lins, m)

    def load_ptq(self, path: str) -> None:
        """Upload the INT8 linears and activation scales of a PTQ artefact
        (no recalibration); the artefact must match this session's shape."""
        from . import ptq
        lins, meta = ptq.load(path)
        by_name = {L.name: L for L in lins}
        c = self.cfg
        if meta.get("n_layers") != c.n_layers or meta.get("d_model") != c.d_model or meta.get("d_ffn") != c.d_ffn:
            raise ValueError("PTQ artefact shape does not match the session")
        scales = np.empty((c.n_layers, 4), np.float32)
        self._bias = []
        for li in range(c.n_layers):
            row = []
            for which, nm in enumerate(self.LINEAR_NAMES):
                L = by_name.get("h.%d.%s" % (li, nm))
                if L is None or L.scales_w is None:
                    raise ValueError("PTQ artefact lacks per-channel linear h.%d.%s" % (li, nm))
                bias = L.bias if L.bias is not None else np.zeros(L.n, np.float32)
                N.call("tvq_session_set_linear_i8", self.handle, li, which, _p(L.w), _p(L.scales_w), _p(bias))
                scales[li, which] = L.scale_a
                row.append(bias)
            self._bias.append(row)
        self.set_act_scales(scales)

    def close(self):
        if getattr(self, "handle", None):
            N.call("tvq_session_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- layout / scales
    def prepare(self, seg, logits_mode: int = 0):
        seg = np.ascontiguousarray(seg, np.int64)
        N.call("tvq_session_prepare", self.handle, _p(seg), seg.size - 1, int(logits_mode))
        self.seg = seg
        self.logits_mode = int(logits_mode)

    @property
    def n_tokens(self) -> int:
        return int(self.seg[-1])

    def act_scales(self) -> np.ndarray:
        out = np.empty(4 * self.cfg.n_layers, np.float32)
        N.call("tvq_session_get_act_scales", self.handle, _p(out), out.size)
        return out.reshape(self.cfg.n_layers, 4)

    def set_act_scales(self, scales):
        s = np.ascontiguousarray(scales, np.float32).ravel()
        N.call("tvq_session_set_act_scales", self.handle, _p(s), s.size)

    def linear_i8(self, layer: int, which: int):
        n, k = {0: (3 * self.cfg.d_model, self.cfg.d_model), 1: (self.cfg.d_model, self.cfg.d_model),
                2: (self.cfg.d_ffn, self.cfg.d_model), 3: (self.cfg.d_model, self.cfg.d_ffn)}[which]
        w = np.empty((n, k), np.int8)
        s = np.empty(n, np.float32)
        N.call("tvq_session_get_linear_i8", self.handle, layer, which, _p(w), _p(s))
        return w, s

    STAGES = ("embed", "layernorm", "gemm_c_attn", "attention", "gemm_attn_proj", "gemm_c_fc", "gemm_mlp_proj",
              "lm_head", "quantize")

    def set_profiling(self, on: bool):
        N.call("tvq_session_set_profiling", self.handle, 1 if on else 0)

    def stage_times(self) -> dict:
        out = np.zeros(len(self.STAGES), np.float32)
        N.call("tvq_session_stage_times", self.handle, _p(out), out.size)
        return dict(zip(self.STAGES, out.tolist()))

    def sync(self):
        N.call("tvq_session_sync", self.handle)

    def launches(self) -> int:
        """Kernel launches of the graph launched last (its kernel nodes)."""
        n = C.c_int64(0)
        N.call("tvq_session_launches", self.handle, C.byref(n))
        return int(n.value)

    def hidden_device_ptr(self) -> int:
        p = C.c_void_p()
        N.call("tvq_session_hidden", self.handle, C.byref(p))
        return p.value

    def run_layers_device(self, x_dev_ptr=None, y_dev_ptr=None, dynamic: bool = False, stream_ptr=None):
        """The blocks alone on device hidden states (asynchronous; ints are
        raw pointers, None = the resident hidden states)."""
        N.call("tvq_session_run_layers", self.handle, C.c_void_p(x_dev_ptr) if x_dev_ptr else None, 1,
               C.c_void_p(y_dev_ptr) if y_dev_ptr else None, 1, 1 if dynamic else 0,
               C.c_void_p(stream_ptr) if stream_ptr else None)


class GPT2Session(_Session):
    """Device-resident INT8 GPT-2 forward on one GPU (one tvq session)."""

    def __init__(self, weights: GPT2Weights, device: int = 0, max_tokens: int = 1024, ptq_path=None):
        """ptq_path: take the blocks' INT8 linears and activation scales from a
        PTQ artefact (export_ptq) instead of quantizing weights' f32 linears."""
        super().__init__(weights.cfg, weights.layers, weights.cfg.vocab, device, max_tokens, ptq_path)
        N.call("tvq_session_set_embeddings", self.handle, _p(_f32(weights.wte)), _p(_f32(weights.wpe)))
        N.call("tvq_session_set_layernorm", self.handle, -1, 0, _p(_f32(weights.lnf_g)), _p(_f32(weights.lnf_b)))

    def logits_shape(self):
        rows = self.n_tokens if self.logits_mode == 0 else self.seg.size - 1
        return rows, self.cfg.vocab

    def calibrate(self, ids, reset: bool = True):
        ids = np.ascontiguousarray(ids, np.int64)
        assert ids.size == self.n_tokens
        N.call("tvq_session_calibrate", self.handle, _p(ids), 0, 1 if reset else 0)

    # ---- forward
    def forward(self, ids) -> np.ndarray:
        """Host ids in, host logits out (synchronous): the reference-facing
        InferenceSession.run equivalent."""
        ids = np.ascontiguousarray(ids, np.int64)
        assert ids.size == self.n_tokens
        rows, V = self.logits_shape()
        out = np.empty((rows, V), np.float32)
        N.call("tvq_session_forward", self.handle, _p(ids), 0, _p(out), out.size, 0, None)
        return out

    def forward_async(self, ids_ptr: int, logits_ptr: int, logits_len: int, stream_ptr=None, ids_on_device=False):
        """Queue a forward whose logits go to host memory and return at once
        (raw pointers: pinned host ids or device ids, pinned host logits of
        at least logits_len floats); wait() before reading the logits.
        Consecutive calls overlap one forward's compute with the previous
        one's logits copy."""
        N.call("tvq_session_forward_async", self.handle, C.c_void_p(ids_ptr), 1 if ids_on_device else 0,
               C.c_void_p(logits_ptr), logits_len, C.c_void_p(stream_ptr) if stream_ptr else None)

    def join(self, stream_ptr=None):
        """The stream waits (the host does not) for every queued logits copy."""
        N.call("tvq_session_join", self.handle, C.c_void_p(stream_ptr) if stream_ptr else None)

    def wait(self, stream_ptr=None):
        """Block until every queued forward and its logits copy are done;
        raises on a device error of those calls."""
        N.call("tvq_session_wait", self.handle, C.c_void_p(stream_ptr) if stream_ptr else None)

    def forward_device(self, ids_dev_ptr=None, logits_dev_ptr=None, stream_ptr=None):
        """Asynchronous forward on device buffers (ints are raw pointers)."""
        N.call("tvq_session_forward", self.handle, C.c_void_p(ids_dev_ptr) if ids_dev_ptr else None, 1,
               C.c_void_p(logits_dev_ptr) if logits_dev_ptr else None, 1 << 62, 1,
               C.c_void_p(stream_ptr) if stream_ptr else None)

    def logits_device_ptr(self) -> int:
        p = C.c_void_p()
        N.call("tvq_session_logits", self.handle, C.byref(p), None, None)
        return p.value



class LayerStack(_Session):
    """The transformer blocks of a GPT2Config without embeddings or LM head:
    hidden states [T, d_model] in, hidden states out (the XL-shaped INT8 PTQ
    layer stack).  With dynamic=True every call calibrates each quantization
    point on its own activations on the GPU (calibrate_minmax +
    quantize_int8_symmetric per layer, engine.tkv:13-36, 216-226)."""

    def __init__(self, cfg: GPT2Config, layers: list, device: int = 0, max_tokens: int = 8192, ptq_path=None):
        super().__init__(cfg, layers, 0, device, max_tokens, ptq_path)

    def run(self, x, dynamic: bool = True) -> np.ndarray:
        """Host hidden states in, host hidden states out (synchronous)."""
        x = _f32(x)
        assert x.shape == (self.n_tokens, self.cfg.d_model)
        y = np.empty_like(x)
        N.call("tvq_session_run_layers", self.handle, _p(x), 0, _p(y), 0, 1 if dynamic else 0, None)
        return y
