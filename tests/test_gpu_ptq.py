"""A GPT-2-shaped session exported as a PTQ artefact (ptq.py) and rebuilt
from it without recalibration: the INT8 linears are the oracle's per-channel
quantization (engine.tkv:202-250) bit for bit, the activation scales are the
session's calibrated ones, and the rebuilt session's logits are the same bits
as the original's."""
import numpy as np
import pytest

from oracle import gpt2_int8 as OG
from tokenvector.inference_b200 import ptq
from tokenvector.inference_b200.gpt2 import GPT2Config, GPT2Session, GPT2Weights, segments_from_lengths

pytestmark = pytest.mark.gpu


def test_export_and_reload_runs_the_same_bits(tmp_path):
    cfg = GPT2Config(vocab=512, d_model=128, n_heads=2, n_layers=2, d_ffn=512, max_pos=1024)
    w = GPT2Weights.random(cfg, seed=13)
    seg = segments_from_lengths([300, 77])
    T = int(seg[-1])
    rng = np.random.default_rng(3)
    calib, ids = rng.integers(0, cfg.vocab, T), rng.integers(0, cfg.vocab, T)
    path = str(tmp_path / "gpt2.tvqptq")
    s = GPT2Session(w, max_tokens=T)
    try:
        s.prepare(seg)
        s.calibrate(calib)
        scales = s.act_scales()
        want = s.forward(ids)
        s.export_ptq(path)
    finally:
        s.close()
    lins, meta = ptq.load(path)
    assert meta["n_layers"] == cfg.n_layers and len(lins) == 4 * cfg.n_layers
    qw = OG.quantize_weights(w.layers)
    for li in range(cfg.n_layers):
        for which in range(4):
            L = lins[4 * li + which]
            assert np.array_equal(L.w, qw[li][which][0])
            assert np.array_equal(L.scales_w.view(np.uint32), qw[li][which][1].view(np.uint32))
            assert ptq.f32_bits(L.scale_a) == ptq.f32_bits(scales[li, which])
    s2 = GPT2Session(w, max_tokens=T, ptq_path=path)
    try:
        s2.prepare(seg)
        assert np.array_equal(s2.act_scales().view(np.uint32), scales.view(np.uint32))
        got = s2.forward(ids)
    finally:
        s2.close()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
