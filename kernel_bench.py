"""Per-kernel timings of libtvq on one GPU (CUDA events, L2 flushed between
repetitions), for tuning and for small profiler captures.

  python kernel_bench.py gemm --m 1024 --n 3072 --k 768 --epilogue gelu_q
  python kernel_bench.py lmhead --m 1024 --n 50257 --k 768
  python kernel_bench.py hbm --m 8192 --n 6400    # calibrate / quantize GB/s
  python kernel_bench.py sweep                     # configs 1 and 3 GEMM shapes
  python kernel_bench.py layernorm --m 1024 --n 768
  python kernel_bench.py attention --m 1024 --n 768 --heads 12
  python kernel_bench.py quantize --m 1024 --n 768
  python kernel_bench.py gpt2       # stage times of the 124M forward
  python kernel_bench.py packed --m 16384 --reps 3   # a config-4-like packed batch, 2 blocks
  python kernel_bench.py all        # the GPT-2 124M shapes
"""
from __future__ import annotations

import argparse
import ctypes as C
import json

import numpy as np

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from tokenvector.inference_b200 import _native as N  # noqa: E402


def _env():
    import torch
    dev = torch.device("cuda:0")
    st = torch.cuda.Stream(dev)
    torch.cuda.set_stream(st)
    flush = _L2Flush(torch, dev)
    return torch, dev, st, flush


class _L2Flush:
    """Between repetitions: write 256 MiB (evicts the timed kernel's data
    from the 126 MB L2), then read another 256 MiB, so that the dirty lines
    of that write are written back before the next timed launch instead of
    during it."""

    def __init__(self, torch, dev):
        self.w = torch.empty(64 << 20, dtype=torch.float32, device=dev)
        self.r = torch.zeros(64 << 20, dtype=torch.float32, device=dev)

    def zero_(self):
        self.w.zero_()
        self.r.sum()


def _time(torch, st, flush, fn, reps):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    tot = 0.0
    for _ in range(reps):
        flush.zero_()
        e0.record(st)
        fn()
        e1.record(st)
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    return 1000.0 * tot / reps  # microseconds


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def bench_gemm(m, n, k, epilogue="f32", reps=20, kind=N.GEMM_I8):
    """epilogue: f32 | f32_residual | gelu_q (GELU-erf then int8 out) |
    gelu_amax (GELU-erf, f32 out and max|y|: a calibrating c_fc)"""
    torch, dev, st, flush = _env()
    dt = torch.int8 if kind == N.GEMM_I8 else torch.uint8
    A = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev).view(dt)
    W = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev).view(dt)
    if kind == N.GEMM_F8:  # finite E4M3 bytes only
        A = (A & 0x77)
        W = (W & 0x77)
    bias = torch.randn(n, device=dev) * 0.02
    sw = torch.rand(n, device=dev) * 0.001
    sa = torch.tensor([0.01], device=dev)
    so = torch.tensor([0.05], device=dev)
    Y = torch.empty((m, n), device=dev) if epilogue != "gelu_q" else None
    Yq = torch.empty((m, n), dtype=torch.int8, device=dev) if epilogue == "gelu_q" else None
    R = torch.randn((m, n), device=dev) if epilogue == "f32_residual" else None
    act = N.ACT_GELU_ERF if epilogue in ("gelu_q", "gelu_amax") else N.ACT_NONE
    amax = torch.zeros(1, dtype=torch.int32, device=dev) if epilogue == "gelu_amax" else None
    sp = C.c_void_p(st.cuda_stream)

    def fn():
        N.call("tvq_dev_gemm", kind, _p(A), _p(W), _p(bias), _p(R), _p(Y), _p(Yq), m, n, k, _p(sa), _p(sw), 1, act,
               _p(so) if Yq is not None else None, _p(amax), sp)
    us = _time(torch, st, flush, fn, reps)
    ops = 2.0 * m * n * k
    byts = m * k + n * k + (4 * m * n if Y is not None else m * n) + (4 * m * n if R is not None else 0) + 8 * n
    out = {"kernel": "gemm", "m": m, "n": n, "k": k, "epilogue": epilogue, "us": us, "tops": ops / us / 1e6,
           "gbs": byts / us / 1e3}
    if m <= 1024:
        out["us_graph"] = _time_graph(torch, st, fn, reps)
    return out


def _time_graph(torch, st, fn, reps, calls=32):
    """Device time per call with the host out of the loop: `calls` calls
    captured in one CUDA graph (their launches back to back, PDL-chained),
    replayed after an L2 flush; inputs stay L2-resident across the calls of
    one replay, as in a decode loop over the same weights."""
    flush = _L2Flush(torch, st.device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for _ in range(calls):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    tot = 0.0
    for _ in range(max(3, reps // 4)):
        flush.zero_()
        e0.record(st)
        g.replay()
        e1.record(st)
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    return 1000.0 * tot / max(3, reps // 4) / calls


def bench_layernorm(m, d, reps=20):
    torch, dev, st, flush = _env()
    x = torch.randn((m, d), device=dev)
    g = torch.ones(d, device=dev)
    b = torch.zeros(d, device=dev)
    q = torch.empty((m, d), dtype=torch.int8, device=dev)
    s = torch.tensor([0.03], device=dev)
    sp = C.c_void_p(st.cuda_stream)
    us = _time(torch, st, flush, lambda: N.call("tvq_dev_layernorm", _p(x), _p(g), _p(b), None, _p(q), _p(s), None,
                                                  m, d, 1e-6, sp), reps)
    return {"kernel": "layernorm_q", "m": m, "d": d, "us": us, "gbs": m * d * 5 / us / 1e3}


def bench_quantize(m, d, reps=20):
    torch, dev, st, flush = _env()
    x = torch.randn((m, d), device=dev)
    q = torch.empty((m, d), dtype=torch.int8, device=dev)
    s = torch.tensor([0.03], device=dev)
    sp = C.c_void_p(st.cuda_stream)
    us = _time(torch, st, flush, lambda: N.call("tvq_dev_quantize_int8", _p(x), _p(q), m * d, _p(s), sp), reps)
    return {"kernel": "quantize_i8", "n": m * d, "us": us, "gbs": m * d * 5 / us / 1e3}


def _peaks():
    import json
    import os
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            m = json.load(f)
        return m["hbm_gbs"], m["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def bench_hbm(m, d, reps=20):
    """The memory-bound calibration / quantize kernels on an [m, d] f32
    tensor larger than L2: GB/s of algorithmic bytes (4 B per element read
    for max-abs, 5 B read + write for the quantizers, + 4 B per row of
    scales) against the measured HBM copy bandwidth."""
    torch, dev, st, flush = _env()
    hbm, _, src = _peaks()
    n = m * d
    x = torch.randn((m, d), device=dev)
    q = torch.empty((m, d), dtype=torch.int8, device=dev)
    mm = torch.empty(2, dtype=torch.int32, device=dev)
    first = torch.empty(1, device=dev)
    s = torch.tensor([0.03], device=dev)
    rs = torch.empty(m, device=dev)
    sp = C.c_void_p(st.cuda_stream)
    cases = [
        # the accumulate launch alone: the running min / max only grows
        ("minmax (calibrate_minmax)", 4 * n,
         lambda: N.call("tvq_dev_minmax_accumulate", _p(x), n, _p(mm), _p(first), sp)),
        ("quantize_i8 per tensor", 5 * n, lambda: N.call("tvq_dev_quantize_int8", _p(x), _p(q), n, _p(s), sp)),
        ("calibrate + quantize per channel (rows)", 5 * n + 4 * m,
         lambda: N.call("tvq_dev_calibrate_quantize_per_channel", _p(x), _p(q), _p(rs), m, d, sp)),
        ("quantize_fp8 e4m3, per-row scale", 5 * n + 4 * m,
         lambda: N.call("tvq_dev_quantize_fp8", _p(x), _p(q), m, d, _p(rs), 2, 0, sp)),
    ]
    out = []
    N.call("tvq_dev_minmax_reset", _p(mm), sp)
    N.call("tvq_dev_calibrate_quantize_per_channel", _p(x), _p(q), _p(rs), m, d, sp)
    for name, byts, fn in cases:
        us = _time(torch, st, flush, fn, reps)
        out.append({"kernel": name, "m": m, "d": d, "us": us, "gbs": byts / us / 1e3,
                    "frac_hbm": byts / us / 1e3 / hbm, "peak_source": "%s HBM copy %.0f GB/s" % (src, hbm)})
    return out


def bench_sweep(reps=20):
    """The quantized GEMM on the BASELINE shapes: config 1 (INT8, M 1024, N
    3072, K 768, per-channel f32 epilogue + bias) and the config-3 FP8 E4M3
    grid ((K, N) in {(1024, 3072), (1024, 4096), (4096, 1024)}, M in {1, 16,
    128, 1024, 8192}); TOPS against 2 x the measured dense bf16 rate."""
    _, bf16, src = _peaks()
    out = []
    r = bench_gemm(1024, 3072, 768, "f32", reps, N.GEMM_I8)
    r.update({"config": 1, "kind": "int8", "frac_peak": r["tops"] / (2 * bf16)})
    out.append(r)
    for (k, n) in [(1024, 3072), (1024, 4096), (4096, 1024)]:
        for m in (1, 16, 128, 1024, 8192):
            r = bench_gemm(m, n, k, "f32", reps, N.GEMM_F8)
            r.update({"config": 3, "kind": "fp8_e4m3", "frac_peak": r["tops"] / (2 * bf16),
                      "peak_source": "2 x %s dense bf16" % src})
            out.append(r)
    return out


def bench_attention(T, d, heads, reps=20):
    torch, dev, st, flush = _env()
    qkv = torch.randn((T, 3 * d), device=dev)
    out = torch.empty((T, d), device=dev)
    tiles = torch.empty((T + 64) * 4, dtype=torch.int32, device=dev)
    seg = np.array([0, T], np.int64)
    sp = C.c_void_p(st.cuda_stream)
    us = _time(torch, st, flush, lambda: N.call("tvq_dev_attention", _p(qkv), seg.ctypes.data_as(C.c_void_p), 1, d,
                                                  heads, _p(tiles), T + 64, _p(out), None, None, None, sp), reps)
    fl = 4.0 * T * T * (d // heads) * heads / 2
    return {"kernel": "attention", "T": T, "d": d, "heads": heads, "us": us, "tflops_causal": fl / us / 1e6}


def bench_lmhead(m, n, k, reps=20):
    """The fp32 tied LM head as the FP16 hi/lo split GEMM (GEMM_F16X3): the
    two row splits once, then Y = A W^T timed alone."""
    torch, dev, st, flush = _env()
    A = torch.randn((m, k), device=dev)
    W = torch.randn((n, k), device=dev) * 0.02
    ah = torch.empty((m, k), dtype=torch.float16, device=dev)
    al = torch.empty_like(ah)
    wh = torch.empty((n, k), dtype=torch.float16, device=dev)
    wl = torch.empty_like(wh)
    ar = torch.empty(m, device=dev)
    wr = torch.empty(n, device=dev)
    Y = torch.empty((m, n), device=dev)
    sp = C.c_void_p(st.cuda_stream)
    N.call("tvq_dev_split_f16_rows", _p(A), _p(ah), _p(al), _p(ar), m, k, sp)
    N.call("tvq_dev_split_f16_rows", _p(W), _p(wh), _p(wl), _p(wr), n, k, sp)
    us = _time(torch, st, flush, lambda: N.call("tvq_dev_gemm_f16x3", _p(ah), _p(al), _p(ar), _p(wh), _p(wl), _p(wr),
                                                  _p(Y), m, n, k, sp), reps)
    ref = (A.double() @ W.double().T)
    err = float(((Y.double() - ref).abs() / (A.double().abs() @ W.double().abs().T)).max())
    return {"kernel": "gemm_f16x3", "m": m, "n": n, "k": k, "us": us,
            "tflops_useful": 2.0 * m * n * k / us / 1e6, "max_err_over_sum_abs": err}


def bench_gpt2(reps=20):
    import torch
    from tokenvector.inference_b200.gpt2 import GPT2Config, GPT2Session, GPT2Weights
    cfg = GPT2Config.gpt2_124m()
    w = GPT2Weights.random(cfg, seed=0)
    s = GPT2Session(w, max_tokens=1024)
    s.prepare(np.array([0, 1024], np.int64))
    s.calibrate(np.random.default_rng(1).integers(0, cfg.vocab, 1024).astype(np.int64))
    _, dev, st, flush = _env()
    ids = torch.randint(0, cfg.vocab, (1024,), dtype=torch.int64, device=dev)
    out = {}
    for prof in (False, True):
        s.set_profiling(prof)
        out["forward_us_profiling" if prof else "forward_us"] = _time(
            torch, st, flush, lambda: s.forward_device(ids.data_ptr(), None, st.cuda_stream), reps)
        if prof:
            out["stages_ms"] = s.stage_times()
    s.close()
    return out


def bench_packed(tokens, layers=2, reps=5):
    """A config-4-like packed batch on GPT-2 124M widths (d 768, 12 heads, ffn
    3072) with `layers` blocks and a small vocabulary: ragged requests of
    U[32, 1024] tokens (seed 7) up to about `tokens`, last-token logits.  One
    calibration forward (eager, general GEMM epilogues), then static-scale
    forwards (CUDA graph) timed with stage events off and on.  Launch order
    for a capture: the calibration forward's kernels, then each forward's
    embed, and per block LayerNorm, c_attn, attention, fix-up, attn c_proj,
    LayerNorm, c_fc, mlp c_proj."""
    import torch
    from tokenvector.inference_b200.gpt2 import GPT2Config, GPT2Session, GPT2Weights, segments_from_lengths
    cfg = GPT2Config(vocab=512, d_model=768, n_heads=12, n_layers=layers, d_ffn=3072, max_pos=1024)
    w = GPT2Weights.random(cfg, seed=1)
    rng = np.random.default_rng(7)
    lengths = []
    while sum(lengths) < tokens - 1024:
        lengths.append(int(rng.integers(32, 1025)))
    seg = segments_from_lengths(lengths)
    T = int(seg[-1])
    s = GPT2Session(w, max_tokens=T)
    s.prepare(seg, logits_mode=1)
    s.calibrate(rng.integers(0, cfg.vocab, T).astype(np.int64))
    _, dev, st, flush = _env()
    ids = torch.randint(0, cfg.vocab, (T,), dtype=torch.int64, device=dev)
    out = {"kernel": "packed", "tokens": T, "requests": len(lengths), "layers": layers}
    for prof in (False, True):
        s.set_profiling(prof)
        out["forward_us_profiling" if prof else "forward_us"] = _time(
            torch, st, flush, lambda: s.forward_device(ids.data_ptr(), None, st.cuda_stream), reps)
        if prof:
            out["stages_ms"] = s.stage_times()
    s.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "lmhead", "hbm", "sweep", "layernorm", "quantize", "attention", "gpt2",
                                     "packed", "all"])
    ap.add_argument("--m", type=int, default=1024)
    ap.add_argument("--n", type=int, default=768)
    ap.add_argument("--k", type=int, default=768)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--epilogue", default="f32", choices=["f32", "f32_residual", "gelu_q", "gelu_amax"])
    ap.add_argument("--fp8", action="store_true")
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    N.lib()
    kind = N.GEMM_F8 if a.fp8 else N.GEMM_I8
    res = []
    if a.what == "gemm":
        res.append(bench_gemm(a.m, a.n, a.k, a.epilogue, a.reps, kind))
    elif a.what == "hbm":
        res.extend(bench_hbm(a.m, a.n, a.reps))
    elif a.what == "sweep":
        res.extend(bench_sweep(a.reps))
    elif a.what == "lmhead":
        res.append(bench_lmhead(a.m, a.n, a.k, a.reps))
    elif a.what == "layernorm":
        res.append(bench_layernorm(a.m, a.n, a.reps))
    elif a.what == "quantize":
        res.append(bench_quantize(a.m, a.n, a.reps))
    elif a.what == "attention":
        res.append(bench_attention(a.m, a.n, a.heads, a.reps))
    elif a.what == "gpt2":
        res.append(bench_gpt2(a.reps))
    elif a.what == "packed":
        res.append(bench_packed(a.m, reps=a.reps))
    else:
        for (n, k, ep) in [(2304, 768, "f32"), (768, 768, "f32_residual"), (3072, 768, "gelu_q"),
                           (768, 3072, "f32_residual")]:
            res.append(bench_gemm(1024, n, k, ep, a.reps))
        for (m, n, k) in [(8192, 6400, 1600), (8192, 8192, 8192)]:
            res.append(bench_gemm(m, n, k, "f32", a.reps))
        res.append(bench_layernorm(1024, 768, a.reps))
        res.append(bench_quantize(1024, 768, a.reps))
        res.append(bench_attention(1024, 768, 12, a.reps))
        res.append(bench_gpt2(a.reps))
    for r in res:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
