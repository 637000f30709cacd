"""GPU parity of the tcgen05 quantized GEMM against the CPU oracle, through
the C ABI: int32 accumulators and fp32 epilogue outputs bit-exact for INT8;
the FP8 path within its stated tolerance."""
import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import _native as N
from tokenvector.inference_b200.quantization import matmul as M

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (3, 5, 7), (1, 64, 16), (17, 33, 100), (128, 128, 128), (130, 250, 300), (200, 96, 768),
          (129, 257, 1040), (64, 2304, 768), (1024, 3072, 768)]


def _mats(m, n, k, seed):
    rng = np.random.default_rng(seed)
    A = rng.integers(-127, 128, (m, k)).astype(np.int8)
    W = rng.integers(-127, 128, (n, k)).astype(np.int8)
    return A, W


def _same(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_int8_accumulators_exact(m, n, k):
    A, W = _mats(m, n, k, m * 7 + n)
    acc = M.gemm_i8_accumulators(A, W, m, n, k)
    assert np.array_equal(acc, O.gemm_i8_acc(A, W))


def test_int8_accumulators_extremes():
    # all +-127: largest |acc| = 16129 * k
    for k in [16, 768, 6400]:
        A = np.full((130, k), -127, np.int8)
        W = np.full((70, k), 127, np.int8)
        W[::2] = -127
        assert np.array_equal(M.gemm_i8_accumulators(A, W, 130, 70, k), O.gemm_i8_acc(A, W))


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_matmul_int8_per_channel_bit_exact(m, n, k):
    A, W = _mats(m, n, k, m + 3 * n + k)
    rng = np.random.default_rng(k)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    sa = np.float32(0.0213)
    sw = (rng.random(n) * 0.003 + 1e-4).astype(np.float32)
    Y = np.empty(m * n, np.float32)
    M.matmul_int8_per_channel(A, W, bias, Y, m, n, k, sa, sw)
    assert _same(Y.reshape(m, n), O.matmul_int8_per_channel(A, W, bias, sa, sw))
    Y2 = np.empty(m * n, np.float32)
    M.matmul_int8_per_channel(A, W, [], Y2, m, n, k, sa, sw)
    assert _same(Y2.reshape(m, n), O.matmul_int8_per_channel(A, W, None, sa, sw))


@pytest.mark.parametrize("m,n,k", SHAPES[:6])
def test_matmul_int8_symmetric_bit_exact(m, n, k):
    A, W = _mats(m, n, k, 99 + m)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    Y = np.empty(m * n, np.float32)
    M.matmul_int8_symmetric(A, W, bias, Y, m, n, k, 0.011, 0.007)
    assert _same(Y.reshape(m, n), O.matmul_int8_symmetric(A, W, bias, 0.011, 0.007))


def test_epilogue_ties_take_the_reference_path():
    # acc odd and above 2^24 sits exactly on a float midpoint: the f32 fast
    # path must defer to the f64 chain (ties to even), per-channel and
    # symmetric, with and without bias.
    k = 1057
    A = np.full((3, k), 127, np.int8)
    W = np.full((4, k), 127, np.int8)
    W[:, -1] = [1, 3, -5, 7]
    acc = O.gemm_i8_acc(A, W)
    assert (acc % 2 == 1).all() and (np.abs(acc) > 2 ** 24).all()
    for bias in (None, np.array([0.0, 1.0, -2.0, 0.5], np.float32)):
        Y = np.empty(12, np.float32)
        M.matmul_int8_per_channel(A, W, bias, Y, 3, 4, k, 1.0, np.ones(4, np.float32))
        assert _same(Y.reshape(3, 4), O.matmul_int8_per_channel(A, W, bias, np.float32(1.0), np.ones(4, np.float32)))
        Y2 = np.empty(12, np.float32)
        M.matmul_int8_symmetric(A, W, bias, Y2, 3, 4, k, 0.5, 2.0)
        assert _same(Y2.reshape(3, 4), O.matmul_int8_symmetric(A, W, bias, np.float32(0.5), np.float32(2.0)))


def test_matmul_k0_is_bias():
    Y = np.empty(6, np.float32)
    bias = np.array([1.5, -2.0, 0.25], np.float32)
    M.matmul_int8_per_channel(np.zeros(0, np.int8), np.zeros(0, np.int8), bias, Y, 2, 3, 0, 0.5,
                              np.ones(3, np.float32))
    assert _same(Y.reshape(2, 3), np.tile(bias, (2, 1)))


def test_matmul_list_i32_form():
    A, W = _mats(9, 11, 40, 1)
    sw = np.full(11, 0.01, np.float32)
    Y = np.empty(99, np.float32)
    M.matmul_int8_per_channel(A.astype(np.int32), W.astype(np.int32), [], Y, 9, 11, 40, 0.02, sw)
    assert _same(Y.reshape(9, 11), O.matmul_int8_per_channel(A, W, None, 0.02, sw))


def test_config1_end_to_end():
    """calibrate (8 batches), quantize X and W, GEMM."""
    from tokenvector.inference_b200.quantization import engine as E
    X = O.gi_noise(1024 * 768, 0, 1.0).reshape(1024, 768)
    Wf = O.gi_noise(3072 * 768, 100).reshape(3072, 768)
    bias = O.gi_noise(3072, 200)
    batches = [X] + [O.gi_noise(1024 * 768, s, 1.0) for s in range(1, 8)]
    p = E.calibrate_minmax_batches(batches, 1)
    op = O.calibrate_minmax(np.concatenate([b.ravel() for b in batches]), 1)
    assert _same(p.scale, op.scale)
    xq = np.empty(X.size, np.int8)
    E.quantize_int8_symmetric(X, xq, p.scale)
    sw = np.array([q.scale for q in E.calibrate_per_channel_minmax(Wf, 3072, 768)], np.float32)
    wq = np.empty(Wf.size, np.int8)
    E.quantize_int8_per_channel(Wf, wq, 3072, 768, sw)
    oxq = O.quantize_int8_symmetric(X, op.scale)
    osw = O.per_channel_scales(Wf, 3072, 768)
    owq = O.quantize_int8_per_channel(Wf, 3072, 768, osw)
    assert np.array_equal(xq.reshape(1024, 768), oxq) and np.array_equal(wq.reshape(3072, 768), owq)
    Y = np.empty(1024 * 3072, np.float32)
    M.matmul_int8_per_channel(xq, wq, bias, Y, 1024, 3072, 768, p.scale, sw)
    assert _same(Y.reshape(1024, 3072), O.matmul_int8_per_channel(oxq, owq, bias, op.scale, osw))


def _fp8_operands(m, n, k, seed):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((m, k)).astype(np.float32)
    idx = rng.choice(m * k, max(1, m * k // 1000), replace=False)
    X.ravel()[idx] *= 20.0
    Wf = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    sa = np.array([np.abs(X).max() / 448.0], np.float32)
    sw = (np.abs(Wf).max(axis=1) / 448.0).astype(np.float32)
    A = O.quantize_fp8_e4m3_scaled(X, sa, False)
    W = O.quantize_fp8_e4m3_scaled(Wf, sw, True)
    return A, W, sa, sw


def _fp8_tol(A, W, sa, sw):
    # |error| <= 2^-20 * sum_k |a_k w_k| * sa * sw[n]  +  the reference's halved
    # subnormals: sum over subnormal operands of |a w| / 2 (types.tkv:221)
    da = np.abs(O.dequantize_fp8_e4m3(A).astype(np.float64))
    dw = np.abs(O.dequantize_fp8_e4m3(W).astype(np.float64))
    mag = da @ dw.T
    sub_a = ((A & 0x78) == 0) & ((A & 0x7) != 0)
    sub_w = ((W & 0x78) == 0) & ((W & 0x7) != 0)
    sub = (da * sub_a) @ dw.T + da @ (dw * sub_w).T
    return (mag * 2.0 ** -20 + sub * 1.01 + 1e-30) * float(sa[0]) * sw.astype(np.float64)[None, :]


@pytest.mark.parametrize("m,n,k", [(1, 3072, 1024), (16, 4096, 1024), (128, 1024, 4096), (300, 200, 160)])
def test_matmul_fp8_within_tolerance(m, n, k):
    A, W, sa, sw = _fp8_operands(m, n, k, m + n)
    bias = np.zeros(n, np.float32)
    Y = np.empty(m * n, np.float32)
    M.matmul_fp8_e4m3(A, W, bias, Y, m, n, k, float(sa[0]), sw)
    ref = O.matmul_fp8_e4m3(A, W, bias, float(sa[0]), sw).astype(np.float64)
    err = np.abs(Y.reshape(m, n).astype(np.float64) - ref)
    tol = _fp8_tol(A, W, sa, sw) + np.abs(ref) * 2.0 ** -23
    assert np.all(err <= tol), float((err / tol).max())


def test_matmul_fp8_unscaled_reference_form():
    # matmul.tkv:46-58: no scales, y = sum dec(a) dec(w) + bias; normal
    # operands only, small K -> exact in fp32 too
    rng = np.random.default_rng(11)
    A = rng.integers(0x08, 0x78, (33, 64)).astype(np.uint8) | (rng.integers(0, 2, (33, 64)) * 0x80).astype(np.uint8)
    W = rng.integers(0x08, 0x40, (17, 64)).astype(np.uint8)
    Y = np.empty(33 * 17, np.float32)
    M.matmul_fp8_e4m3(A.astype(np.int32) - 128, W.astype(np.int32) - 128, [], Y, 33, 17, 64)
    ref = O.matmul_fp8_e4m3(A, W, None).astype(np.float64)
    err = np.abs(Y.reshape(33, 17).astype(np.float64) - ref)
    tol = _fp8_tol(A, W, np.ones(1, np.float32), np.ones(17, np.float32)) + np.abs(ref) * 2.0 ** -23
    assert np.all(err <= tol)


def test_gemm_errors():
    with pytest.raises(ValueError):
        M.matmul_int8_per_channel(np.zeros(8, np.int8), np.zeros(12, np.int8), [], np.zeros(6, np.float32),
                                  2, 3, 4, 1.0, np.ones(2, np.float32))
    with pytest.raises(ValueError):
        M.matmul_int8_per_channel(np.zeros(8, np.int8), np.zeros(12, np.int8), np.ones(2, np.float32),
                                  np.zeros(6, np.float32), 2, 3, 4, 1.0, np.ones(3, np.float32))


def test_device_gemm_fused_epilogue():
    """tvq_dev_gemm with GELU + residual + int8 output + amax on torch tensors."""
    import torch
    m, n, k = 256, 384, 512
    A, W = _mats(m, n, k, 5)
    rng = np.random.default_rng(5)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    sw = (rng.random(n) * 0.002 + 1e-4).astype(np.float32)
    R = rng.standard_normal((m, n)).astype(np.float32)
    dev = torch.device("cuda:0")
    tA, tW = torch.from_numpy(A).to(dev), torch.from_numpy(W).to(dev)
    tb, tsw = torch.from_numpy(bias).to(dev), torch.from_numpy(sw).to(dev)
    tR = torch.from_numpy(R).to(dev)
    sa = torch.tensor([0.03], dtype=torch.float32, device=dev)
    so = torch.tensor([0.05], dtype=torch.float32, device=dev)
    Y = torch.empty((m, n), dtype=torch.float32, device=dev)
    Yq = torch.empty((m, n), dtype=torch.int8, device=dev)
    amax = torch.zeros(1, dtype=torch.int32, device=dev)
    from tokenvector.inference_b200.quantization import _buf as B
    N.call("tvq_dev_gemm", N.GEMM_I8, B.ptr(tA), B.ptr(tW), B.ptr(tb), B.ptr(tR), B.ptr(Y), B.ptr(Yq), m, n, k,
           B.ptr(sa), B.ptr(tsw), 1, N.ACT_GELU_ERF, B.ptr(so), B.ptr(amax), B.stream_of(tA))
    torch.cuda.synchronize()
    base = O.matmul_int8_per_channel(A, W, bias, np.float32(0.03), sw)
    gel = O.gelu_erf_array(base)
    want = O.add(gel, R)
    got = Y.cpu().numpy()
    assert np.allclose(got, want, rtol=2e-6, atol=2e-6)
    q_ref = O.quantize_int8_symmetric(got, np.float32(0.05))
    assert np.array_equal(Yq.cpu().numpy(), q_ref)
    am = amax.cpu().numpy().view(np.float32)[0]
    assert am == np.abs(got).max()


@pytest.mark.parametrize("m,n,k", [(1, 50257, 768), (37, 1000, 64), (1024, 4096, 768), (130, 300, 1600)])
def test_split_tf32_gemm_is_fp32_accurate(m, n, k):
    """The LM head's fp32 GEMM on tensor cores (hi/lo split on the TF32 grid:
    22-bit operands, 3 products): |error| <= 2^-18 * sum_k |a_k w_k| per
    output against a float64 reference, and within 4x the max error of
    torch's true-fp32 (non-TF32) matmul on the same data."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    rng = np.random.default_rng(m + n)
    A = rng.standard_normal((m, k)).astype(np.float32)
    W = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    dev = torch.device("cuda:0")
    tA, tW = torch.from_numpy(A).to(dev), torch.from_numpy(W).to(dev)
    parts = [torch.empty_like(t) for t in (tA, tA, tW, tW)]
    from tokenvector.inference_b200.quantization import _buf as B
    N.call("tvq_dev_split_tf32", B.ptr(tA), B.ptr(parts[0]), B.ptr(parts[1]), tA.numel(), None)
    N.call("tvq_dev_split_tf32", B.ptr(tW), B.ptr(parts[2]), B.ptr(parts[3]), tW.numel(), None)
    Y = torch.empty((m, n), dtype=torch.float32, device=dev)
    N.call("tvq_dev_gemm_f32x3", *(B.ptr(p) for p in parts), B.ptr(Y), m, n, k, None)
    torch.cuda.synchronize()
    # the split represents x to 2^-22 relative
    d = (parts[0].double() + parts[1].double() - tA.double()).abs()
    assert bool((d <= tA.double().abs() * 2.0 ** -22).all())
    ref = A.astype(np.float64) @ W.astype(np.float64).T
    mag = np.abs(A).astype(np.float64) @ np.abs(W).astype(np.float64).T
    err = np.abs(Y.cpu().numpy().astype(np.float64) - ref)
    t32 = (tA @ tW.T).cpu().numpy().astype(np.float64)
    e32 = np.abs(t32 - ref)
    assert np.all(err <= mag * 2.0 ** -18 + 1e-30), float((err / (mag + 1e-30)).max())
    assert err.max() <= 4.0 * e32.max() + 1e-12, (err.max(), e32.max())


def _split_f16(t):
    """Row-scaled fp16 split through the C-ABI: (hi, lo, rscale)."""
    import torch
    from tokenvector.inference_b200.quantization import _buf as B
    rows, k = t.shape
    hi = torch.empty((rows, k), dtype=torch.float16, device=t.device)
    lo = torch.empty_like(hi)
    rs = torch.empty((rows,), dtype=torch.float32, device=t.device)
    N.call("tvq_dev_split_f16_rows", B.ptr(t), B.ptr(hi), B.ptr(lo), B.ptr(rs), rows, k, None)
    return hi, lo, rs


def test_split_f16_rows_represents_rows_to_2e22():
    """hi + lo under the row's power-of-two scale: the largest |x*s| sits in
    [2^14, 2^15), |x*s - hi - lo| <= max(2^-22 |x*s|, 2^-25); zero rows get
    scale 1; rows of very different magnitude get their own scales."""
    import torch
    rng = np.random.default_rng(7)
    X = rng.standard_normal((64, 200)).astype(np.float32)
    X[1] *= 1e-20
    X[2] *= 1e20
    X[3] = 0.0
    X[4, 5] = 3.0e38
    X[5] = np.ldexp(rng.standard_normal(200), rng.integers(-60, 1, 200)).astype(np.float32)
    t = torch.from_numpy(X).cuda()
    hi, lo, rs = _split_f16(t)
    torch.cuda.synchronize()
    s = 1.0 / rs.double().cpu().numpy()
    xs = X.astype(np.float64) * s[:, None]
    h, l = hi.double().cpu().numpy(), lo.double().cpu().numpy()
    assert np.all(np.abs(xs - h - l) <= np.maximum(np.abs(xs) * 2.0 ** -22, 2.0 ** -25))
    mx = np.abs(xs).max(axis=1)
    nz = mx > 0
    assert np.all((mx[nz] >= 2.0 ** 14) & (mx[nz] < 2.0 ** 15))
    assert s[3] == 1.0
    assert np.all(np.log2(s) == np.round(np.log2(s)))


@pytest.mark.parametrize("m,n,k", [(1, 50257, 768), (37, 1000, 64), (1024, 4096, 768), (130, 300, 1600),
                                   (200, 129, 8)])
def test_f16_split_gemm_is_fp32_accurate(m, n, k):
    """The LM head's fp32 GEMM on the FP16 tensor cores (row-scaled fp16
    hi/lo split, 3 products, power-of-two scales undone in the epilogue):
    |error| <= 2^-18 * sum_k |a_k w_k| per output against a float64
    reference, and at most the larger of 4x the max error of torch's
    true-fp32 (non-TF32) matmul on the same data and 2^-22 * sum_k |a_k w_k|
    (the split operands' own precision; torch's one-row GEMV sums more
    exactly than a GEMM).  Rows of A span 2^-30..2^30 in magnitude."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    rng = np.random.default_rng(m + n + k)
    A = rng.standard_normal((m, k)).astype(np.float32)
    A *= np.ldexp(1.0, rng.integers(-30, 31, (m, 1))).astype(np.float32)
    W = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    dev = torch.device("cuda:0")
    tA, tW = torch.from_numpy(A).to(dev), torch.from_numpy(W).to(dev)
    ah, al, ar = _split_f16(tA)
    wh, wl, wr = _split_f16(tW)
    from tokenvector.inference_b200.quantization import _buf as B
    Y = torch.empty((m, n), dtype=torch.float32, device=dev)
    N.call("tvq_dev_gemm_f16x3", B.ptr(ah), B.ptr(al), B.ptr(ar), B.ptr(wh), B.ptr(wl), B.ptr(wr), B.ptr(Y),
           m, n, k, None)
    torch.cuda.synchronize()
    ref = A.astype(np.float64) @ W.astype(np.float64).T
    mag = np.abs(A).astype(np.float64) @ np.abs(W).astype(np.float64).T
    err = np.abs(Y.cpu().numpy().astype(np.float64) - ref)
    t32 = (tA @ tW.T).cpu().numpy().astype(np.float64)
    e32 = np.abs(t32 - ref) / (mag + 1e-300)
    rel = err / (mag + 1e-300)
    assert np.all(rel <= 2.0 ** -18), float(rel.max())
    assert rel.max() <= max(4.0 * e32.max(), 2.0 ** -22), (rel.max(), e32.max())


def test_matmul_fp8_config3_grid_worst_error(capsys):
    """BASELINE config 3 (FP8 E4M3 PTQ GEMM, GPT-2-medium widths): activations
    N(0,1) with 0.1 % outliers x20, weights N(0,0.02), per-tensor / per-channel
    scales amax/448.  Over the (K, N) grid and M up to 1024, the worst error
    relative to sum |a w| sa sw, the fraction of E4M3 subnormal operands, and
    the share of the tolerance the OCP-vs-reference subnormal decode takes;
    every element within the stated tolerance."""
    lines = []
    for (k, n) in [(1024, 3072), (1024, 4096), (4096, 1024)]:
        for m in (1, 16, 128, 1024):
            A, W, sa, sw = _fp8_operands(m, n, k, 7 * m + n + k)
            Y = np.empty(m * n, np.float32)
            M.matmul_fp8_e4m3(A, W, None, Y, m, n, k, float(sa[0]), sw)
            ref = O.matmul_fp8_e4m3(A, W, None, float(sa[0]), sw).astype(np.float64)
            err = np.abs(Y.reshape(m, n).astype(np.float64) - ref)
            tol = _fp8_tol(A, W, sa, sw) + np.abs(ref) * 2.0 ** -23
            assert np.all(err <= tol), (m, n, k, float((err / tol).max()))
            da = np.abs(O.dequantize_fp8_e4m3(A).astype(np.float64))
            dw = np.abs(O.dequantize_fp8_e4m3(W).astype(np.float64))
            mag = (da @ dw.T) * float(sa[0]) * sw.astype(np.float64)[None, :]
            sub_a = float((((A & 0x78) == 0) & ((A & 0x7) != 0)).mean())
            sub_w = float((((W & 0x78) == 0) & ((W & 0x7) != 0)).mean())
            lines.append("fp8 config3 m=%d n=%d k=%d: max err/sum|aw| %.3g, max err/tol %.3g, subnormal bytes "
                         "A %.2f%% W %.2f%%" % (m, n, k, float((err / (mag + 1e-30)).max()),
                                                  float((err / tol).max()), 100 * sub_a, 100 * sub_w))
    with capsys.disabled():
        print("\n" + "\n".join(lines))


def _dev_gemm(tA, tW, tb, tR, Y, Yq, m, n, k, sa, tsw, per_channel, act, so):
    from tokenvector.inference_b200.quantization import _buf as B
    N.call("tvq_dev_gemm", N.GEMM_I8, B.ptr(tA), B.ptr(tW), B.ptr(tb), B.ptr(tR), B.ptr(Y), B.ptr(Yq), m, n, k,
           B.ptr(sa), B.ptr(tsw), per_channel, act, B.ptr(so), 0, B.stream_of(tA))


@pytest.mark.parametrize("m,n,k,seed,nonfinite", [(1024, 3072, 768, 11, False), (200, 320, 768, 12, True),
                                                  (130, 4096, 1600, 13, False), (1, 64, 16, 14, True),
                                                  (300, 6400, 1600, 15, False)])
def test_device_gemm_gelu_int8_only_exact(m, n, k, seed, nonfinite):
    """GELU-erf -> int8 with no f32 output (the c_fc form of a static-scale
    forward): every int8 is the reference's quantize (engine.tkv:216-226) of
    the reference's GELU (tensor.tkv:165-190) of the reference's dequant
    (matmul.tkv:28), elements near an int8 rounding boundary, saturated ones
    and non-finite biases included."""
    import torch
    A, W = _mats(m, n, k, seed)
    rng = np.random.default_rng(seed)
    bias = (rng.standard_normal(n) * 0.5).astype(np.float32)
    if nonfinite:
        bias[:3] = [np.inf, -np.inf, np.nan]
    sw = (rng.random(n) * 2e-4 + 1e-5).astype(np.float32)
    sa_v, so_v = np.float32(0.05), np.float32(0.03)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    tA, tW, tb, tsw = t(A), t(W), t(bias), t(sw)
    sa = torch.tensor([sa_v], dtype=torch.float32, device=dev)
    so = torch.tensor([so_v], dtype=torch.float32, device=dev)
    Yq = torch.empty((m, n), dtype=torch.int8, device=dev)
    _dev_gemm(tA, tW, tb, None, None, Yq, m, n, k, sa, tsw, 1, N.ACT_GELU_ERF, so)
    torch.cuda.synchronize()
    base = O.matmul_int8_per_channel(A, W, bias, sa_v, sw)
    want = O.quantize_int8_symmetric(O.gelu_erf_array(base), so_v)
    got = Yq.cpu().numpy()
    bad = np.argwhere(got != want)
    assert bad.size == 0, "%d int8 values differ, first at %s: %d vs %d" % (
        len(bad), tuple(bad[0]), got[tuple(bad[0])], want[tuple(bad[0])])
    # the data reach the saturation bound and the rounding boundaries
    assert (np.abs(want) == 127).any()


@pytest.mark.parametrize("m,n,k,in_place", [(1024, 768, 3072, True), (1024, 768, 768, False), (77, 1600, 6400, True),
                                            (300, 512, 64, False), (129, 4096, 1040, True)])
def test_device_gemm_residual_f32_exact(m, n, k, in_place):
    """Dequant + bias + residual with an f32 output only (the c_proj form of a
    forward, the residual stream updated in place): fl32 of the reference's
    f64 chain plus the residual, bit for bit."""
    import torch
    A, W = _mats(m, n, k, 21)
    rng = np.random.default_rng(21)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    sw = (rng.random(n) * 2e-4 + 1e-5).astype(np.float32)
    R = rng.standard_normal((m, n)).astype(np.float32)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    tA, tW, tb, tsw, tR = t(A), t(W), t(bias), t(sw), t(R)
    sa = torch.tensor([0.02], dtype=torch.float32, device=dev)
    Y = tR if in_place else torch.empty((m, n), dtype=torch.float32, device=dev)
    _dev_gemm(tA, tW, tb, tR, Y, None, m, n, k, sa, tsw, 1, N.ACT_NONE, None)
    torch.cuda.synchronize()
    want = O.add(O.matmul_int8_per_channel(A, W, bias, np.float32(0.02), sw), R)
    assert _same(Y.cpu().numpy(), want)


@pytest.mark.parametrize("m,n,k", [(1024, 3072, 768), (300, 6400, 1600), (1, 64, 16)])
def test_device_gemm_gelu_f32_amax(m, n, k):
    """GELU-erf with an f32 output and max |y| (the c_fc of a calibrating
    forward and of per-call calibration): the outputs within the fast GELU's
    tolerance of the reference GELU of the reference dequant, and the
    recorded max |y| equal to the largest |y| written."""
    import torch
    from tokenvector.inference_b200.quantization import _buf as B
    A, W = _mats(m, n, k, 31)
    rng = np.random.default_rng(31)
    bias = (rng.standard_normal(n) * 0.5).astype(np.float32)
    sw = (rng.random(n) * 2e-4 + 1e-5).astype(np.float32)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    tA, tW, tb, tsw = t(A), t(W), t(bias), t(sw)
    sa = torch.tensor([0.05], dtype=torch.float32, device=dev)
    Y = torch.empty((m, n), dtype=torch.float32, device=dev)
    amax = torch.zeros(1, dtype=torch.int32, device=dev)
    N.call("tvq_dev_gemm", N.GEMM_I8, B.ptr(tA), B.ptr(tW), B.ptr(tb), None, B.ptr(Y), None, m, n, k,
           B.ptr(sa), B.ptr(tsw), 1, N.ACT_GELU_ERF, None, B.ptr(amax), B.stream_of(tA))
    torch.cuda.synchronize()
    want = O.gelu_erf_array(O.matmul_int8_per_channel(A, W, bias, np.float32(0.05), sw))
    got = Y.cpu().numpy()
    assert np.allclose(got, want, rtol=2e-6, atol=2e-6)
    assert amax.cpu().numpy().view(np.float32)[0] == np.abs(got).max()
