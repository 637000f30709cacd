"""GPT-2 INT8 PTQ forward on the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Composition of the restated reference functions (oracle/tvq_oracle.c) in the
shape of tv/training/gpt2_ref.tkv:575-610 with the four linears of every
block as QuantizedGemm (tv/runtime/session.tkv:678-697):

  x = embed(ids, pos)                                    gpt2_ref.tkv:80-88
  per layer:
    a  = layernorm(x)                 -> q0 = quantize_int8_symmetric(a, s0)
    qkv = matmul_int8_per_channel(q0, Wqkv, b, s0, sw)   matmul.tkv:17-29
    ctx = causal attention(qkv)       -> q1 = quantize(ctx, s1)
    x  = x + matmul_int8_per_channel(q1, Wproj, ...)
    m  = layernorm(x)                 -> q2 = quantize(m, s2)
    g  = gelu_erf(matmul_int8_per_channel(q2, Wfc, ...)) -> q3 = quantize(g, s3)
    x  = x + matmul_int8_per_channel(q3, Wmp, ...)
  logits = layernorm_f(x) @ wte^T

Weights are quantized per output channel (calibrate_per_channel_minmax +
quantize_int8_per_channel on W^T).  With calibrate=True each activation
scale s_i is calibrate_minmax(activation).scale (engine.tkv:13-36) taken
over all batches seen so far (running max), and used immediately.
"""
from __future__ import annotations

import numpy as np

from . import (add, attention_causal, calibrate_minmax, embed, gelu_erf_array, layernorm, lm_head,
               matmul_int8_per_channel, per_channel_scales, quantize_int8_per_channel, quantize_int8_symmetric)

LINEARS = (("attn_w", "attn_b"), ("proj_w", "proj_b"), ("fc_w", "fc_b"), ("mp_w", "mp_b"))


def quantize_weights(layers):
    """Per-output-channel INT8 of every linear: list of 4-tuples (Wq [n,k], sw [n])."""
    out = []
    for L in layers:
        q = []
        for wk, _ in LINEARS:
            wt = np.ascontiguousarray(np.asarray(L[wk], np.float32).T)  # [k,n] -> [n,k]
            n, k = wt.shape
            sw = per_channel_scales(wt, n, k)
            q.append((quantize_int8_per_channel(wt, n, k, sw), sw))
        out.append(q)
    return out


def positions(seg):
    seg = np.asarray(seg, np.int64)
    pos = np.empty(int(seg[-1]), np.int64)
    for s in range(seg.size - 1):
        pos[seg[s]:seg[s + 1]] = np.arange(seg[s + 1] - seg[s])
    return pos


class Calibrator:
    """Running max|x| per quantization point across calibration batches."""

    def __init__(self, n_layers):
        self.amax = np.zeros((n_layers, 4), np.float64)

    def scale(self, layer, point, x):
        x = np.asarray(x, np.float32)
        # calibrate_minmax(symmetric) over the union of batches seen so far
        am = float(np.max(np.abs(x[~np.isnan(x)]))) if x.size else 0.0
        self.amax[layer, point] = max(self.amax[layer, point], am)
        cat = np.array([self.amax[layer, point]], np.float32)
        return np.float32(calibrate_minmax(cat, 1).scale)

    def scales(self):
        return np.array([[calibrate_minmax(np.array([a], np.float32), 1).scale for a in row] for row in self.amax],
                        np.float32)


def blocks(layers, x, seg, scales=None, calibrator: Calibrator | None = None, qweights=None, n_heads: int = 12,
           eps: float = 1e-6, record=None):
    """The transformer blocks (gpt2_ref.tkv:575-588 per layer) on hidden
    states x f32 [T, d]; returns the new hidden states.  Exactly one of
    `scales` ([L,4] static) or `calibrator` must be given.  `record`: a list
    that receives one dict of every intermediate per layer, or a callable
    record(layer, dict) (then nothing is kept)."""
    assert (scales is None) != (calibrator is None)
    seg = np.asarray(seg, np.int64)
    if qweights is None:
        qweights = quantize_weights(layers)
    x = np.asarray(x, np.float32)
    for li, L in enumerate(layers):
        (wq0, sw0), (wq1, sw1), (wq2, sw2), (wq3, sw3) = qweights[li]

        def sc(point, act):
            return calibrator.scale(li, point, act) if calibrator is not None else np.float32(scales[li][point])

        x_in = x
        a = layernorm(x, L["ln1_g"], L["ln1_b"], eps)
        s0 = sc(0, a)
        q0 = quantize_int8_symmetric(a, s0)
        qkv = matmul_int8_per_channel(q0, wq0, L["attn_b"], s0, sw0)
        ctx = attention_causal(qkv, n_heads, seg)
        s1 = sc(1, ctx)
        q1 = quantize_int8_symmetric(ctx, s1)
        proj = matmul_int8_per_channel(q1, wq1, L["proj_b"], s1, sw1)
        x = add(x, proj)
        x_mid = x
        m = layernorm(x, L["ln2_g"], L["ln2_b"], eps)
        s2 = sc(2, m)
        q2 = quantize_int8_symmetric(m, s2)
        fc = matmul_int8_per_channel(q2, wq2, L["fc_b"], s2, sw2)
        g = gelu_erf_array(fc)
        s3 = sc(3, g)
        q3 = quantize_int8_symmetric(g, s3)
        mp = matmul_int8_per_channel(q3, wq3, L["mp_b"], s3, sw3)
        x = add(x, mp)
        if record is not None:
            rec = dict(x_in=x_in, a=a, s0=s0, q0=q0, qkv=qkv, ctx=ctx, s1=s1, q1=q1, proj=proj, x_mid=x_mid, m=m,
                       s2=s2, q2=q2, fc=fc, g=g, s3=s3, q3=q3, mp=mp, x=x)
            if callable(record):
                record(li, rec)
            else:
                record.append(rec)
    return x


def forward(weights, ids, seg, scales=None, calibrator: Calibrator | None = None, qweights=None,
            logits_mode: int = 0, n_heads: int = 12, eps: float = 1e-6, record=None):
    """INT8 forward.  `weights`: object with wte, wpe, lnf_g, lnf_b, layers
    (dicts as in tokenvector.inference_b200.gpt2.GPT2Weights).  Exactly one of
    `scales` ([L,4] static) or `calibrator` must be given.  Returns logits
    (all rows, or the last row of each sequence for logits_mode 1)."""
    seg = np.asarray(seg, np.int64)
    x = embed(ids, positions(seg), weights.wte, weights.wpe)
    x = blocks(weights.layers, x, seg, scales, calibrator, qweights, n_heads, eps, record)
    xf = layernorm(x, weights.lnf_g, weights.lnf_b, eps)
    if logits_mode == 1:
        xf = np.ascontiguousarray(xf[seg[1:] - 1])
    return lm_head(xf, weights.wte)
