"""GPU parity of the group-wise INT4 path (tv/quantization/int4.tkv) against
the oracle: the codecs bit-exact (packed bytes, scales, zero points,
dequantized values), permute_cols exact, and the grouped GEMM on the tensor
cores within |error| <= 2^-18 * sum_k |a_k w_k| of the oracle's f64 sum
(fp32 accuracy: fp16 hi/lo activations, exact integer weights, per-group
promotion), through both the device and the host-buffer C-ABI forms."""
import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import _native as N
from tokenvector.inference_b200.quantization import _buf as B
from tokenvector.inference_b200.quantization import int4 as Q4

pytestmark = pytest.mark.gpu


def _data(rows, cols, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, cols)) * rng.choice([1e-3, 0.02, 1.0, 30.0], (rows, 1))).astype(np.float32)
    x[0, : min(cols, 8)] = 0.0                       # a zero run (1e-8 floor when a whole group)
    x[min(1, rows - 1), ::3] = np.round(x[min(1, rows - 1), ::3] * 4) / 4  # ties
    if rows > 2:
        x[2] = np.abs(x[2]) + 1.0                    # an all-positive row (asym zp = 0 branch)
    if rows > 3:
        x[3] = -np.abs(x[3]) - 1.0                   # an all-negative row (zp = 15)
    return x


@pytest.mark.parametrize("rows,cols,gs", [(1, 16, 16), (7, 64, 32), (64, 768, 128), (33, 96, 6), (300, 512, 64)])
def test_int4_codecs_bit_exact(rows, cols, gs):
    import torch
    x = _data(rows, cols, rows + cols)
    pk, sc = O.quantize_int4_grouped(x, rows, cols, gs)
    tx = torch.from_numpy(x).cuda()
    gpk, gsc = Q4.quantize_int4_grouped(tx, rows, cols, gs)
    assert np.array_equal(gpk.cpu().numpy(), pk.ravel())
    assert np.array_equal(gsc.cpu().numpy().view(np.uint32), sc.ravel().view(np.uint32))
    deq = Q4.dequantize_int4_grouped(gpk, None, rows, cols, gs, gsc)
    assert np.array_equal(deq.cpu().numpy().view(np.uint32),
                          O.dequantize_int4_grouped(pk, rows, cols, gs, sc).ravel().view(np.uint32))
    pk, sc, zp = O.quantize_int4_grouped_asym(x, rows, cols, gs)
    gpk, gsc, gzp = Q4.quantize_int4_grouped_asym(tx, rows, cols, gs)
    assert np.array_equal(gpk.cpu().numpy(), pk.ravel())
    assert np.array_equal(gzp.cpu().numpy(), zp.ravel())
    assert np.array_equal(gsc.cpu().numpy().view(np.uint32), sc.ravel().view(np.uint32))
    deq = Q4.dequantize_int4_grouped_asym(gpk, None, rows, cols, gs, gsc, gzp)
    assert np.array_equal(deq.cpu().numpy().view(np.uint32),
                          O.dequantize_int4_grouped_asym(pk, rows, cols, gs, sc, zp).ravel().view(np.uint32))
    # host-buffer forms give the same bytes
    hpk, hsc = Q4.quantize_int4_grouped(x, rows, cols, gs)
    assert np.array_equal(hpk, O.quantize_int4_grouped(x, rows, cols, gs)[0].ravel())


def test_permute_cols_and_errors():
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 37)).astype(np.float32)
    perm = rng.permutation(37).astype(np.int64)
    ref = O.permute_cols(x, 5, 37, perm)
    got = Q4.permute_cols(torch.from_numpy(x).cuda(), 5, 37, torch.from_numpy(perm).cuda())
    assert np.array_equal(got.cpu().numpy(), ref.ravel())
    back = Q4.inv_permute_cols(got, 5, 37, torch.from_numpy(perm).cuda())
    assert np.array_equal(back.cpu().numpy(), x.ravel())
    assert np.array_equal(Q4.inv_permute_cols(Q4.permute_cols(x, 5, 37, perm), 5, 37, perm), x.ravel())
    with pytest.raises(ValueError):
        Q4.permute_cols(x, 5, 37, perm[:36])
    bad = perm.copy()
    bad[4] = 37
    with pytest.raises(N.TvqError):  # an index out of range is reported, not read
        Q4.permute_cols(x, 5, 37, bad)
    with pytest.raises(ValueError):
        Q4.quantize_int4_grouped(x.ravel(), 5, 37, 37)  # odd cols


def _gemm_case(m, n, k, gs, seed, perm=False, bias=True):
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((m, k)) * np.ldexp(1.0, rng.integers(-10, 11, (m, 1)))).astype(np.float32)
    W = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    pk, sc = O.quantize_int4_grouped(W, n, k, gs)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32) if bias else np.zeros(0, np.float32)
    pm = rng.permutation(k).astype(np.int64) if perm else None
    return A, pk, sc, b, pm


def _bound(A, pk, sc, n, k, gs, pm):
    Wd = O.dequantize_int4_grouped(pk, n, k, gs, sc).astype(np.float64)
    Ad = A.astype(np.float64)
    if pm is not None:
        Ad = Ad[:, pm]
    return np.abs(Ad) @ np.abs(Wd).T


@pytest.mark.parametrize("m,n,k,gs,perm", [(1, 64, 128, 32, False), (37, 300, 256, 64, False),
                                           (128, 512, 1024, 128, False), (200, 129, 96, 32, True),
                                           (64, 256, 768, 16, True), (1024, 2304, 768, 128, False)])
def test_matmul_int4_grouped_fp32_accurate(m, n, k, gs, perm):
    import torch
    A, pk, sc, b, pm = _gemm_case(m, n, k, gs, m + n + k, perm)
    ref = O.matmul_int4_grouped(A, pk, b, gs, sc, pm).astype(np.float64)
    dev = torch.device("cuda:0")
    Y = torch.empty((m, n), dtype=torch.float32, device=dev)
    tA, tpk, tsc = torch.from_numpy(A).to(dev), torch.from_numpy(pk.ravel()).to(dev), torch.from_numpy(sc).to(dev)
    tb = torch.from_numpy(b).to(dev)
    tpm = torch.from_numpy(pm).to(dev) if pm is not None else None
    if perm:
        Q4.matmul_int4_grouped_ordered(tA, tpk, tb, Y, m, n, k, gs, tsc, tpm)
    else:
        Q4.matmul_int4_grouped(tA, tpk, tb, Y, m, n, k, gs, tsc)
    torch.cuda.synchronize()
    got = Y.cpu().numpy().astype(np.float64)
    mag = _bound(A, pk, sc, n, k, gs, pm) + np.abs(b)[None, :]
    err = np.abs(got - ref)
    assert np.all(err <= mag * 2.0 ** -18 + 1e-30), float((err / (mag + 1e-30)).max())
    # the host-buffer form (the reference's call shape) agrees bit for bit
    if m * n <= 40000:
        py = np.empty(m * n, np.float32)
        if perm:
            Q4.matmul_int4_grouped_ordered(A, pk, b, py, m, n, k, gs, sc, pm)
        else:
            Q4.matmul_int4_grouped(A, pk, b, py, m, n, k, gs, sc)
        assert np.array_equal(py.view(np.uint32), Y.cpu().numpy().ravel().view(np.uint32))


def test_matmul_int4_edges():
    import torch
    # k = 0: the bias alone; empty bias
    y = np.empty(3 * 4, np.float32)
    Q4.matmul_int4_grouped(np.zeros(0, np.float32), np.zeros(0, np.uint8), np.arange(4, dtype=np.float32), y,
                           3, 4, 0, 16, np.zeros(0, np.float32))
    assert np.array_equal(y.reshape(3, 4), np.tile(np.arange(4, dtype=np.float32), (3, 1)))
    A, pk, sc, b, _ = _gemm_case(5, 7, 64, 16, 9, bias=False)
    py = np.empty(35, np.float32)
    Q4.matmul_int4_grouped(A, pk, b, py, 5, 7, 64, 16, sc)
    ref = O.matmul_int4_grouped(A, pk, b, 16, sc).astype(np.float64).ravel()
    mag = _bound(A, pk, sc, 7, 64, 16, None).ravel()
    assert np.all(np.abs(py - ref) <= mag * 2.0 ** -18 + 1e-30)
    with pytest.raises(ValueError):
        Q4.matmul_int4_grouped(A, pk, b, py, 5, 7, 64, 16, sc[:, :1])  # scales_w too small
    with pytest.raises(ValueError):
        Q4.matmul_int4_grouped(A, pk, b, py, 5, 7, 64, 24, sc)        # k not a multiple of group_size
