"""Parity at the benchmark configurations' own shapes (4
and 5), against the CPU oracle composition of the reference functions
(oracle/gpt2_int8.py: gpt2_ref.tkv:575-610 with the four linears of every
block as QuantizedGemm, session.tkv:678-697).

* Layer by layer at the GPT-2 124M shape (12 layers, d 768, 12 heads, seq
  1024): every GPU stage is fed the ORACLE's own input for that stage, so
  nothing upstream can differ.  Bit-exact: the quantized weights and scales,
  the int32 accumulators of all four GEMMs, their fp32 outputs (dequant +
  bias, + residual for the two projections, c_fc before its GELU), and every
  int8 activation: the attention context's (the tensor-core kernel plus its
  f64 fix-up of undecided rows) and the GELU output's (exact GELU where the
  int8 rounding is undecided).  Within a stated tolerance: LayerNorm (f64
  statistics summed as a tree instead of in sequence: within 1 ulp on at
  most 1e-5 of the elements; its int8 output within 1 step on the same
  fraction and always the exact quantize of its own f32 output), the f32
  attention context (rtol 1e-4, atol 2e-6 against the f64 oracle) and the
  f32 GELU (rtol 2e-6, atol 2e-6).  Each layer's four calibrated scales from
  the GPU's max |x| on the oracle's activations equal the oracle's to 1e-5.
* Whole models with the oracle's static scales: since every int8 activation
  is the reference's, the hidden states after the last block are the
  oracle's bit for bit (config 2's 12 layers at seq 1024, a config-4 sample
  of four ragged requests, config 5's XL-width blocks), and the logits
  differ only by the fp32 LM head's own error (within 2^-18 sum|x w| per
  logit, bounded here by 1e-4).
* Calibrating runs (the calibration forward; config 5's per-call
  calibration): their f32 attention / GELU outputs and max |x| are the fast
  kernels' (within the tolerances above), so a scale can differ from the
  oracle's in its last bits; quantizing with it then moves int8 values that
  lie within that difference of a rounding boundary, and such a change
  propagates to the later layers.  Those runs keep bounds measured at these
  shapes (B200): scales within 2e-2 relative (largest seen 6e-3); three
  XL-width blocks with per-call calibration: mean |diff| 1.7e-2, largest
  0.126 on hidden states of unit scale, bounded here by 3e-2 and 0.2.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from oracle import gpt2_int8 as OG
from tokenvector.inference_b200 import _native as N
from tokenvector.inference_b200.gpt2 import (GPT2Config, GPT2Session, GPT2Weights, LayerStack, gi_noise,
                                             random_layers, segments_from_lengths)

pytestmark = pytest.mark.gpu

SEQ = 1024


def _up(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _flip_stats(got, ref):
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    rowmax = diff.max(axis=1)
    return float(diff.mean()), float((rowmax > 2e-3).mean()), float(rowmax.max())


def _assert_flip_bounded(got, ref, rows_frac):
    mean, frac, worst = _flip_stats(got, ref)
    assert mean < 2e-4 and frac <= rows_frac and worst < 5e-2, dict(mean=mean, rows_above_2e3=frac, worst=worst)


@pytest.fixture(scope="module")
def gpt2_124m():
    """The config-2 model: GPT-2 124M, the reference's LCG + Box-Muller init
    (gpt2_ref.tkv:1977-2026), seed 0 as bench.py; the oracle's per-channel
    INT8 weights; a calibration sequence and an input sequence."""
    cfg = GPT2Config.gpt2_124m()
    w = GPT2Weights.random(cfg, seed=0)
    qw = OG.quantize_weights(w.layers)
    calib_ids = np.random.default_rng(1).integers(0, cfg.vocab, SEQ).astype(np.int64)
    ids = np.random.default_rng(2).integers(0, cfg.vocab, SEQ).astype(np.int64)
    seg = np.array([0, SEQ], np.int64)
    cal = OG.Calibrator(cfg.n_layers)
    x0 = O.embed(calib_ids, OG.positions(seg), w.wte, w.wpe)
    OG.blocks(w.layers, x0, seg, calibrator=cal, qweights=qw, n_heads=cfg.n_heads, eps=cfg.eps)
    return dict(cfg=cfg, w=w, qw=qw, calib_ids=calib_ids, ids=ids, seg=seg, scales=cal.scales())


class _LayerChecker:
    """GPU stages of one block fed with the oracle's intermediates."""

    def __init__(self, cfg, layers, qw, seg):
        import torch
        self.torch = torch
        self.cfg, self.layers, self.qw, self.seg = cfg, layers, qw, seg
        self.fail = []
        self.ln_mismatch = []

    def _gemm(self, A, W, bias, sa, sw, residual=None, act=N.ACT_NONE):
        torch = self.torch
        m, k = A.shape
        n = W.shape[0]
        tA, tW, tb, tsw = _up(A), _up(W), _up(bias), _up(sw)
        ts = _up(np.array([sa], np.float32))
        tR = _up(residual) if residual is not None else None
        Y = torch.empty((m, n), dtype=torch.float32, device="cuda:0")
        N.call("tvq_dev_gemm", N.GEMM_I8, _p(tA), _p(tW), _p(tb), _p(tR), _p(Y), None, m, n, k, _p(ts), _p(tsw), 1,
               act, None, None, None)
        torch.cuda.synchronize()
        return Y.cpu().numpy()

    def _acc(self, A, W):
        m, k = A.shape
        n = W.shape[0]
        acc = np.empty((m, n), np.int32)
        A = np.ascontiguousarray(A)
        W = np.ascontiguousarray(W)
        N.call("tvq_gemm_i8_acc", A.ctypes.data_as(C.c_void_p), W.ctypes.data_as(C.c_void_p),
               acc.ctypes.data_as(C.c_void_p), m, n, k)
        return acc

    def _ln(self, x, g, b, s):
        torch = self.torch
        T, d = x.shape
        tx, tg, tb = _up(x), _up(g), _up(b)
        ts = _up(np.array([s], np.float32))
        y = torch.empty((T, d), dtype=torch.float32, device="cuda:0")
        q = torch.empty((T, d), dtype=torch.int8, device="cuda:0")
        N.call("tvq_dev_layernorm", _p(tx), _p(tg), _p(tb), _p(y), _p(q), _p(ts), None, T, d, self.cfg.eps, None)
        torch.cuda.synchronize()
        return y.cpu().numpy(), q.cpu().numpy()

    def _quant(self, x, s):
        torch = self.torch
        tx = _up(x)
        q = torch.empty(x.shape, dtype=torch.int8, device="cuda:0")
        ts = _up(np.array([s], np.float32))
        N.call("tvq_dev_quantize_int8", _p(tx), _p(q), x.size, _p(ts), None)
        torch.cuda.synchronize()
        return q.cpu().numpy()

    def _attention(self, qkv, s1=None):
        """f32 context, and with a scale the int8 context of the same call
        (tensor-core kernel + exact fix-up) and the amax of the f32 one."""
        torch = self.torch
        T = qkv.shape[0]
        d = self.cfg.d_model
        tq = _up(qkv)
        out = torch.empty((T, d), dtype=torch.float32, device="cuda:0")
        cap = 2 * (T // 64 + 2 * (self.seg.size - 1))
        tiles = torch.empty(cap * 4, dtype=torch.int32, device="cuda:0")
        q = ts = None
        if s1 is not None:
            q = torch.empty((T, d), dtype=torch.int8, device="cuda:0")
            ts = _up(np.array([s1], np.float32))
        am = torch.zeros(1, dtype=torch.int32, device="cuda:0")
        N.call("tvq_dev_attention", _p(tq), self.seg.ctypes.data_as(C.c_void_p), self.seg.size - 1, d,
               self.cfg.n_heads, _p(tiles), cap, _p(out), _p(q), _p(ts), _p(am), None)
        torch.cuda.synchronize()
        return out.cpu().numpy(), (q.cpu().numpy() if q is not None else None), am.cpu().numpy().view(np.float32)[0]

    def _gelu_q(self, A, W, bias, sa, sw, so):
        """c_fc with GELU-erf -> int8 (the session's form) and, apart, the
        max |GELU| of a calibrating run (f32 output + amax)."""
        torch = self.torch
        m, k = A.shape
        n = W.shape[0]
        tA, tW, tb, tsw = _up(A), _up(W), _up(bias), _up(sw)
        ts, tso = _up(np.array([sa], np.float32)), _up(np.array([so], np.float32))
        Yq = torch.empty((m, n), dtype=torch.int8, device="cuda:0")
        N.call("tvq_dev_gemm", N.GEMM_I8, _p(tA), _p(tW), _p(tb), None, None, _p(Yq), m, n, k, _p(ts), _p(tsw), 1,
               N.ACT_GELU_ERF, _p(tso), None, None)
        Y = torch.empty((m, n), dtype=torch.float32, device="cuda:0")
        am = torch.zeros(1, dtype=torch.int32, device="cuda:0")
        N.call("tvq_dev_gemm", N.GEMM_I8, _p(tA), _p(tW), _p(tb), None, _p(Y), None, m, n, k, _p(ts), _p(tsw), 1,
               N.ACT_GELU_ERF, None, _p(am), None)
        torch.cuda.synchronize()
        return Yq.cpu().numpy(), Y.cpu().numpy(), am.cpu().numpy().view(np.float32)[0]

    def _ln_amax(self, x, g, b):
        torch = self.torch
        T, d = x.shape
        tx, tg, tb = _up(x), _up(g), _up(b)
        y = torch.empty((T, d), dtype=torch.float32, device="cuda:0")
        am = torch.zeros(1, dtype=torch.int32, device="cuda:0")
        N.call("tvq_dev_layernorm", _p(tx), _p(tg), _p(tb), _p(y), None, None, _p(am), T, d, self.cfg.eps, None)
        torch.cuda.synchronize()
        return am.cpu().numpy().view(np.float32)[0]

    def _check(self, li, what, ok):
        if not ok:
            self.fail.append("layer %d: %s" % (li, what))

    def _check_ln(self, li, what, y, q, ref_y, ref_q, s):
        ulps = np.abs(y.view(np.int32).astype(np.int64) - ref_y.view(np.int32).astype(np.int64))
        qd = np.abs(q.astype(np.int32) - ref_q.astype(np.int32))
        self.ln_mismatch.append(int((ulps > 0).sum()))
        self._check(li, what + " f32 within 1 ulp on <= 1e-5", ulps.max() <= 1 and (ulps > 0).mean() <= 1e-5)
        self._check(li, what + " int8 within 1 on <= 1e-5", qd.max() <= 1 and (qd > 0).mean() <= 1e-5)
        self._check(li, what + " int8 = quantize(own f32)", np.array_equal(q, O.quantize_int8_symmetric(y, s)))

    def _check_scale(self, li, what, gpu_amax, ref_tensor):
        """calibrate_minmax(symmetric) of the GPU's max |x| against the
        oracle's calibrate_minmax of its own tensor (engine.tkv:13-36)."""
        g = np.float32(max(float(gpu_amax), 1e-8) / 127.0)
        r = np.float32(O.calibrate_minmax(ref_tensor, 1).scale)
        self._check(li, what + " calibrated scale within 1e-5", abs(float(g) - float(r)) <= 1e-5 * float(r))

    def __call__(self, li, r):
        L = self.layers[li]
        (wq0, sw0), (wq1, sw1), (wq2, sw2), (wq3, sw3) = self.qw[li]
        y, q = self._ln(r["x_in"], L["ln1_g"], L["ln1_b"], r["s0"])
        self._check_ln(li, "ln_1", y, q, r["a"], r["q0"], r["s0"])
        self._check_scale(li, "ln_1", self._ln_amax(r["x_in"], L["ln1_g"], L["ln1_b"]), r["a"])
        # c_attn: int32 accumulators and fp32 dequant + bias, bit for bit
        self._check(li, "c_attn int32 accumulators", np.array_equal(self._acc(r["q0"], wq0), O.gemm_i8_acc(r["q0"], wq0)))
        self._check(li, "c_attn f32 output", _same_bits(self._gemm(r["q0"], wq0, L["attn_b"], r["s0"], sw0), r["qkv"]))
        ctx, cq, cam = self._attention(r["qkv"], r["s1"])
        self._check(li, "attention within rtol 1e-4 / atol 2e-6", np.allclose(ctx, r["ctx"], rtol=1e-4, atol=2e-6))
        self._check(li, "int8 attention context (kernel + exact fix-up)", np.array_equal(cq, r["q1"]))
        self._check_scale(li, "attention", cam, r["ctx"])
        self._check(li, "int8 of the oracle's context", np.array_equal(self._quant(r["ctx"], r["s1"]), r["q1"]))
        self._check(li, "attn c_proj int32 accumulators",
                    np.array_equal(self._acc(r["q1"], wq1), O.gemm_i8_acc(r["q1"], wq1)))
        self._check(li, "attn c_proj f32 output", _same_bits(self._gemm(r["q1"], wq1, L["proj_b"], r["s1"], sw1), r["proj"]))
        self._check(li, "attn c_proj + residual",
                    _same_bits(self._gemm(r["q1"], wq1, L["proj_b"], r["s1"], sw1, residual=r["x_in"]), r["x_mid"]))
        y, q = self._ln(r["x_mid"], L["ln2_g"], L["ln2_b"], r["s2"])
        self._check_ln(li, "ln_2", y, q, r["m"], r["q2"], r["s2"])
        self._check_scale(li, "ln_2", self._ln_amax(r["x_mid"], L["ln2_g"], L["ln2_b"]), r["m"])
        self._check(li, "c_fc int32 accumulators", np.array_equal(self._acc(r["q2"], wq2), O.gemm_i8_acc(r["q2"], wq2)))
        self._check(li, "c_fc f32 output", _same_bits(self._gemm(r["q2"], wq2, L["fc_b"], r["s2"], sw2), r["fc"]))
        gq, g, gam = self._gelu_q(r["q2"], wq2, L["fc_b"], r["s2"], sw2, r["s3"])
        self._check(li, "GELU within 2e-6", np.allclose(g, r["g"], rtol=2e-6, atol=2e-6))
        self._check(li, "int8 GELU output (exact where undecided)", np.array_equal(gq, r["q3"]))
        self._check_scale(li, "GELU", gam, r["g"])
        self._check(li, "mlp c_proj int32 accumulators",
                    np.array_equal(self._acc(r["q3"], wq3), O.gemm_i8_acc(r["q3"], wq3)))
        self._check(li, "mlp c_proj f32 output", _same_bits(self._gemm(r["q3"], wq3, L["mp_b"], r["s3"], sw3), r["mp"]))
        self._check(li, "mlp c_proj + residual",
                    _same_bits(self._gemm(r["q3"], wq3, L["mp_b"], r["s3"], sw3, residual=r["x_mid"]), r["x"]))


def _hidden(sess, T, d):
    """The session's resident hidden states [T, d] after its last run."""
    from cuda.bindings import runtime as rt
    out = np.empty((T, d), np.float32)
    sess.sync()
    (err,) = rt.cudaMemcpy(out.ctypes.data, sess.hidden_device_ptr(), out.nbytes,
                           rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess
    return out


def _assert_logits_close(got, ref):
    """Logits of identical hidden states: only the fp32 LM head's own error."""
    assert got.shape == ref.shape and np.isfinite(got).all()
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    assert diff.max() <= 1e-4, (float(diff.max()), float(diff.mean()))


def test_config2_weights_and_calibration(gpt2_124m):
    """The 48 INT8 linears equal the oracle's per-channel quantization bit
    for bit; the GPU calibration forward's scales against the oracle's
    (calibrating runs: module docstring)."""
    M = gpt2_124m
    cfg = M["cfg"]
    s = GPT2Session(M["w"], max_tokens=SEQ)
    try:
        for li in range(cfg.n_layers):
            for which in range(4):
                gw, gs = s.linear_i8(li, which)
                assert np.array_equal(gw, M["qw"][li][which][0]), (li, which)
                assert _same_bits(gs, M["qw"][li][which][1]), (li, which)
        s.prepare(M["seg"])
        s.calibrate(M["calib_ids"])
        g = s.act_scales()
    finally:
        s.close()
    rel = np.abs(g.astype(np.float64) - M["scales"]) / M["scales"]
    assert np.allclose(g[0, 0], M["scales"][0, 0], rtol=1e-5, atol=0)  # nothing upstream of the first LayerNorm
    assert rel.max() <= 2e-2, rel.max()


def test_config2_every_layer_bit_exact_on_the_oracles_inputs(gpt2_124m):
    """All 12 blocks of GPT-2 124M at seq 1024, each GPU stage on the
    oracle's own input for it (module docstring)."""
    M = gpt2_124m
    cfg, w = M["cfg"], M["w"]
    chk = _LayerChecker(cfg, w.layers, M["qw"], M["seg"])
    x = O.embed(M["ids"], OG.positions(M["seg"]), w.wte, w.wpe)
    OG.blocks(w.layers, x, M["seg"], scales=M["scales"], qweights=M["qw"], n_heads=cfg.n_heads, eps=cfg.eps,
              record=chk)
    assert not chk.fail, chk.fail[:20]
    # LayerNorm is the only stage allowed to differ; report how often it did
    assert sum(chk.ln_mismatch) <= 1e-5 * 2 * cfg.n_layers * SEQ * cfg.d_model


def test_config2_whole_forward_bit_exact_hidden_states(gpt2_124m):
    """The whole 12-layer forward on the device session with the oracle's
    static scales: hidden states after the last block bit for bit, all
    1024 x 50257 logits within the LM head's fp32 error."""
    M = gpt2_124m
    cfg, w = M["cfg"], M["w"]
    s = GPT2Session(w, max_tokens=SEQ)
    try:
        s.prepare(M["seg"])
        s.set_act_scales(M["scales"])
        got = s.forward(M["ids"])
        hid = _hidden(s, SEQ, cfg.d_model)
    finally:
        s.close()
    x = O.embed(M["ids"], OG.positions(M["seg"]), w.wte, w.wpe)
    href = OG.blocks(w.layers, x, M["seg"], scales=M["scales"], qweights=M["qw"], n_heads=cfg.n_heads, eps=cfg.eps)
    nbad = int((hid.view(np.uint32) != href.view(np.uint32)).sum())
    assert nbad == 0, (nbad, float(np.abs(hid - href).max()))
    ref = O.lm_head(O.layernorm(href, w.lnf_g, w.lnf_b, cfg.eps), w.wte)
    _assert_logits_close(got, ref)


def test_config4_ragged_sample(gpt2_124m):
    """Config 4's serving layout on a sample: four packed requests of
    lengths 1024, 517, 33 and 300 (the block-diagonal causal mask of
    pack_rows / pack_block_mask, session.tkv:3506-3566) with the oracle's
    scales of a calibration pass on the same layout: hidden states bit for
    bit, all-token logits within the LM head's error, and the last-token
    logits (what config 4 serves) equal to those rows."""
    M = gpt2_124m
    cfg, w = M["cfg"], M["w"]
    lengths = [1024, 517, 33, 300]
    seg = segments_from_lengths(lengths)
    T = int(seg[-1])
    rng = np.random.default_rng(44)
    calib = rng.integers(0, cfg.vocab, T).astype(np.int64)
    ids = rng.integers(0, cfg.vocab, T).astype(np.int64)
    cal = OG.Calibrator(cfg.n_layers)
    OG.blocks(w.layers, O.embed(calib, OG.positions(seg), w.wte, w.wpe), seg, calibrator=cal, qweights=M["qw"],
              n_heads=cfg.n_heads, eps=cfg.eps)
    scales = cal.scales()
    s = GPT2Session(w, max_tokens=T)
    try:
        s.prepare(seg, logits_mode=0)
        s.set_act_scales(scales)
        got = s.forward(ids)
        hid = _hidden(s, T, cfg.d_model)
        s.prepare(seg, logits_mode=1)
        last = s.forward(ids)
    finally:
        s.close()
    x = O.embed(ids, OG.positions(seg), w.wte, w.wpe)
    href = OG.blocks(w.layers, x, seg, scales=scales, qweights=M["qw"], n_heads=cfg.n_heads, eps=cfg.eps)
    nbad = int((hid.view(np.uint32) != href.view(np.uint32)).sum())
    assert nbad == 0, (nbad, float(np.abs(hid - href).max()))
    _assert_logits_close(got, O.lm_head(O.layernorm(href, w.lnf_g, w.lnf_b, cfg.eps), w.wte))
    assert last.shape == (4, cfg.vocab)
    assert np.allclose(last, got[seg[1:] - 1], rtol=1e-5, atol=1e-6)


def test_config4_large_packed_batch_grouped_fixup():
    """A packed batch large enough (13,312 tokens x 12 heads) that the exact
    int8 fix-up of the attention context runs several rows per CTA at once
    (the row-group form of a config-4 step): GPT-2 124M widths, two blocks,
    ragged requests of 32 to 1024 tokens, the oracle's scales of a calibration pass on the same
    layout; hidden states after both blocks bit for bit."""
    import torch
    cfg = GPT2Config(vocab=512, d_model=768, n_heads=12, n_layers=2, d_ffn=3072, max_pos=1024)
    w = GPT2Weights.random(cfg, seed=5)
    qw = OG.quantize_weights(w.layers)
    rng = np.random.default_rng(45)
    lengths = []
    while sum(lengths) < 13312 - 1056:
        lengths.append(int(rng.integers(32, 1025)))
    lengths += [(13312 - sum(lengths)) // 2, 13312 - sum(lengths) - (13312 - sum(lengths)) // 2]
    assert sum(lengths) == 13312 and all(32 <= v <= 1024 for v in lengths), lengths
    seg = segments_from_lengths(lengths)
    T = int(seg[-1])
    assert T * cfg.n_heads >= 1024 * torch.cuda.get_device_properties(0).multi_processor_count
    calib = rng.integers(0, cfg.vocab, T).astype(np.int64)
    ids = rng.integers(0, cfg.vocab, T).astype(np.int64)
    cal = OG.Calibrator(cfg.n_layers)
    OG.blocks(w.layers, O.embed(calib, OG.positions(seg), w.wte, w.wpe), seg, calibrator=cal, qweights=qw,
              n_heads=cfg.n_heads, eps=cfg.eps)
    scales = cal.scales()
    s = GPT2Session(w, max_tokens=T)
    try:
        s.prepare(seg, logits_mode=1)
        s.set_act_scales(scales)
        s.forward(ids)
        hid = _hidden(s, T, cfg.d_model)
    finally:
        s.close()
    x = O.embed(ids, OG.positions(seg), w.wte, w.wpe)
    href = OG.blocks(w.layers, x, seg, scales=scales, qweights=qw, n_heads=cfg.n_heads, eps=cfg.eps)
    nbad = int((hid.view(np.uint32) != href.view(np.uint32)).sum())
    assert nbad == 0, (nbad, float(np.abs(hid - href).max()))


def test_config5_three_xl_blocks_two_sequences():
    """Config 5's layer stack at the XL widths (d 1600, 25 heads, ffn 6400):
    three blocks on two 1024-token sequences of N(0,1) hidden states.  Every
    activation calibrated on the GPU per call (config 5's mode) against the
    oracle with its own calibrator (calibrating-run bounds, module
    docstring); then with those scales as static ones, bit for bit."""
    cfg = GPT2Config(vocab=0, d_model=1600, n_heads=25, n_layers=3, d_ffn=6400, max_pos=1024)
    layers = random_layers(cfg, seed=21)
    seg = segments_from_lengths([SEQ, SEQ])
    T = int(seg[-1])
    x = gi_noise(T * cfg.d_model, 5, 1.0).reshape(T, cfg.d_model)
    qw = OG.quantize_weights(layers)
    st = LayerStack(cfg, layers, max_tokens=T)
    try:
        st.prepare(seg)
        for li in range(cfg.n_layers):
            for which in range(4):
                gw, gs = st.linear_i8(li, which)
                assert np.array_equal(gw, qw[li][which][0]) and _same_bits(gs, qw[li][which][1])
        got = st.run(x, dynamic=True)
        gscales = st.act_scales()
        cal = OG.Calibrator(cfg.n_layers)
        ref = OG.blocks(layers, x, seg, calibrator=cal, qweights=qw, n_heads=cfg.n_heads)
        rel = np.abs(gscales.astype(np.float64) - cal.scales()) / cal.scales()
        assert rel.max() <= 2e-2, rel.max()
        mean, frac, worst = _flip_stats(got, ref)
        assert mean < 3e-2 and worst < 0.2, (mean, frac, worst)
        # static scales: every int8 activation the reference's
        st.set_act_scales(cal.scales())
        got_s = st.run(x, dynamic=False)
        ref_s = OG.blocks(layers, x, seg, scales=cal.scales(), qweights=qw, n_heads=cfg.n_heads)
        nbad = int((got_s.view(np.uint32) != ref_s.view(np.uint32)).sum())
        assert nbad == 0, (nbad, float(np.abs(got_s - ref_s).max()))
    finally:
        st.close()
