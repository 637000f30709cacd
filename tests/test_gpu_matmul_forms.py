"""The two remaining quantized GEMM forms of tv/quantization/matmul.tkv on
the tensor cores, against the oracle's restatements:

  matmul_int8_asymmetric (:31-44)  bit-exact (zero points in the epilogue)
  matmul_fp16 (:79-96)             within (k/16 + 2) 2^-23 sum_k |a w| + 2^-24 |y|
  quantize_fp16 (:106-114)         bit-exact (the reference's encoder)
"""
import numpy as np
import pytest
import torch

import oracle as O
from tokenvector.inference_b200 import _native as N
from tokenvector.inference_b200.quantization import matmul as QM

pytestmark = pytest.mark.gpu


def _i8(rng, shape):
    return rng.integers(-128, 128, shape).astype(np.int8)


@pytest.mark.parametrize("m,n,k,zpa,zpw", [(1, 64, 768, 3, -5), (130, 300, 200, -128, 127),
                                           (1024, 768, 3072, 17, 2), (64, 96, 512, 1 << 17, -(1 << 17)),
                                           (33, 48, 16, 0, 0)])
def test_matmul_int8_asymmetric_bit_exact(m, n, k, zpa, zpw):
    rng = np.random.default_rng(m + n + k)
    A, W = _i8(rng, (m, k)), _i8(rng, (n, k))
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    sa, sw = np.float32(0.0123), np.float32(0.00457)
    y = np.empty(m * n, np.float32)
    QM.matmul_int8_asymmetric(A, W, bias, y, m, n, k, float(sa), zpa, float(sw), zpw)
    ref = O.matmul_int8_asymmetric(A, W, bias, sa, zpa, sw, zpw)
    assert np.array_equal(y.reshape(m, n).view(np.uint32), ref.view(np.uint32))


def test_matmul_int8_asymmetric_list_storage_device_and_edges():
    rng = np.random.default_rng(3)
    m, n, k = 40, 72, 96
    A, W = _i8(rng, (m, k)), _i8(rng, (n, k))
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    ref = O.matmul_int8_asymmetric(A, W, bias, np.float32(0.02), -7, np.float32(0.003), 9)
    # the reference's list[i32] storage
    y = np.empty(m * n, np.float32)
    QM.matmul_int8_asymmetric(A.astype(np.int32), W.astype(np.int32), bias, y, m, n, k, 0.02, -7, 0.003, 9)
    assert np.array_equal(y.reshape(m, n).view(np.uint32), ref.view(np.uint32))
    ai, wi = A.astype(np.int32), W.astype(np.int32)
    yi = np.empty(m * n, np.float32)
    N.call("tvq_matmul_int8_asymmetric_i32", ai.ctypes.data, wi.ctypes.data, bias.ctypes.data, n, yi.ctypes.data, m, n,
           k, 0.02, -7, 0.003, 9)
    assert np.array_equal(yi.reshape(m, n).view(np.uint32), ref.view(np.uint32))
    # device buffers
    dev = torch.device("cuda", 0)
    yd = torch.empty((m, n), dtype=torch.float32, device=dev)
    QM.matmul_int8_asymmetric(torch.from_numpy(A).to(dev), torch.from_numpy(W).to(dev), torch.from_numpy(bias).to(dev),
                              yd, m, n, k, 0.02, -7, 0.003, 9)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    # k = 0: the bias alone
    y0 = np.empty(m * n, np.float32)
    QM.matmul_int8_asymmetric(np.zeros((m, 0), np.int8), np.zeros((n, 0), np.int8), bias, y0, m, n, 0, 0.02, 5, 0.003, 6)
    assert np.array_equal(y0.reshape(m, n), np.broadcast_to(bias, (m, n)))
    # zero points whose corrected sums could leave binary64's exact range
    with pytest.raises(N.TvqError):
        QM.matmul_int8_asymmetric(A, W, bias, y, m, n, k, 0.02, (1 << 17) + 1, 0.003, 0)


def _f16(rng, shape, scale):
    return O.quantize_fp16((rng.standard_normal(shape) * scale).astype(np.float32))


def _fp16_bound(A, W, k, ref):
    fa = np.array([O.f16_decode(v) for v in range(65536)], np.float64)
    s = np.abs(fa[A]) @ np.abs(fa[W]).T
    return (k / 16 + 2) * 2.0 ** -23 * s + 2.0 ** -24 * np.abs(ref)


@pytest.mark.parametrize("m,n,k", [(2, 2, 2), (1, 3072, 1024), (128, 4096, 1024), (300, 200, 104)])
def test_matmul_fp16_within_bound(m, n, k):
    rng = np.random.default_rng(m * n + k)
    A, W = _f16(rng, (m, k), 1.0), _f16(rng, (n, k), 0.02)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    y = np.empty(m * n, np.float32)
    QM.matmul_fp16(A, W, bias, y, m, n, k)
    ref = O.matmul_fp16(A, W, bias)
    err = np.abs(y.reshape(m, n).astype(np.float64) - ref)
    bound = _fp16_bound(A, W, k, ref)
    assert (err <= bound).all(), float((err / bound).max())


def test_matmul_fp16_subnormal_operands():
    # W entirely in fp16's subnormal range (|w| < 2^-14): the products are
    # exact in fp32 and must not be flushed
    m, n, k = 64, 128, 256
    rng = np.random.default_rng(11)
    A = _f16(rng, (m, k), 1.0)
    W = _f16(rng, (n, k), 2e-6)
    assert (((W & 0x7C00) == 0)).all()
    y = np.empty(m * n, np.float32)
    QM.matmul_fp16(A, W, None, y, m, n, k)
    ref = O.matmul_fp16(A, W, None)
    err = np.abs(y.reshape(m, n).astype(np.float64) - ref)
    assert (err <= _fp16_bound(A, W, k, ref)).all()


def test_matmul_fp16_known_answer_list_storage_and_device():
    # inference_tests.tkv:656-664 through the reference's byte lists
    qa = np.zeros(8, np.int32)
    QM.quantize_fp16(np.array([1.0, 0.0, 0.0, 1.0], np.float32), qa)
    y2 = np.zeros(4, np.float32)
    QM.matmul_fp16(qa, qa, np.zeros(2, np.float32), y2, 2, 2, 2)
    assert abs(y2[0] - 1.0) < 0.001 and abs(y2[3] - 1.0) < 0.001
    assert qa.tolist() == [0, 60, 0, 0, 0, 0, 0, 60]  # 0x3C00 as (low, high) signed bytes
    # device buffers, k a multiple of 8
    m, n, k = 96, 160, 64
    rng = np.random.default_rng(2)
    A, W = _f16(rng, (m, k), 1.0), _f16(rng, (n, k), 0.05)
    dev = torch.device("cuda", 0)
    yd = torch.empty((m, n), dtype=torch.float32, device=dev)
    QM.matmul_fp16(torch.from_numpy(A.view(np.int16)).to(dev), torch.from_numpy(W.view(np.int16)).to(dev), None, yd,
                   m, n, k)
    torch.cuda.synchronize()
    ref = O.matmul_fp16(A, W, None)
    err = np.abs(yd.cpu().numpy().astype(np.float64) - ref)
    assert (err <= _fp16_bound(A, W, k, ref)).all()


def test_quantize_fp16_bit_exact():
    # every high half-word with 16 low half-words around the rounding points,
    # plus random patterns: all exponent classes, ties, subnormal carries
    hi = np.arange(65536, dtype=np.uint32) << 16
    lows = np.array([0, 1, 0x0FFF, 0x1000, 0x1001, 0x1FFF, 0x2000, 0x3000, 0x5000, 0x7FFF, 0x8000, 0x8001,
                     0xA000, 0xC000, 0xEFFF, 0xFFFF], np.uint32)
    bits = (hi[:, None] | lows[None, :]).ravel()
    bits = np.concatenate([bits, np.random.default_rng(0).integers(0, 1 << 32, 1 << 22, dtype=np.uint64)
                           .astype(np.uint32)])
    x = bits.view(np.float32)
    ref = O.quantize_fp16(x)
    q = np.empty(x.size, np.uint16)
    QM.quantize_fp16(x, q)
    assert np.array_equal(q, ref)
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    qd = torch.empty(x.size, dtype=torch.int16, device=dev)
    N.call("tvq_dev_quantize_fp16", xd.data_ptr(), qd.data_ptr(), x.size, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(qd.cpu().numpy().view(np.uint16), ref)
