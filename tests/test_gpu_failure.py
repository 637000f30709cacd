"""Failure detection on the GPU without a fault: every tensor-core kernel
bounds its mbarrier waits (a %globaltimer limit, then an error code in the
device error word and a normal exit).  tvq_selftest_wait_timeout makes one
such wait run out on a barrier that nothing arrives at; the call must report
TVQ_ERR_TIMEOUT, the error word must be cleared by that report, and the next
GEMM on the same device must still be bit-exact against the oracle."""
import time

import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import _native as N
from tokenvector.inference_b200.quantization import matmul as M

pytestmark = pytest.mark.gpu


def _gemm_bit_exact(seed):
    rng = np.random.default_rng(seed)
    m, n, k = 130, 200, 256
    A = rng.integers(-127, 128, (m, k)).astype(np.int8)
    W = rng.integers(-127, 128, (n, k)).astype(np.int8)
    bias = rng.standard_normal(n).astype(np.float32)
    sw = (rng.random(n) * 0.01).astype(np.float32)
    Y = np.empty(m * n, np.float32)
    M.matmul_int8_per_channel(A, W, bias, Y, m, n, k, 0.02, sw)
    ref = O.matmul_int8_per_channel(A, W, bias, np.float32(0.02), sw)
    return np.array_equal(Y.reshape(m, n).view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("limit_us", [1000, 5000])
def test_bounded_wait_times_out_and_device_stays_usable(limit_us):
    import torch
    torch.cuda.set_device(0)
    assert _gemm_bit_exact(1)
    t0 = time.perf_counter()
    rc = N.lib().tvq_selftest_wait_timeout(limit_us, None)
    dt = time.perf_counter() - t0
    assert rc == N.TVQ_ERR_TIMEOUT, (rc, N.last_error())
    assert "timed out" in N.last_error()
    # the wait gave up after its limit (plus one check period), not at once
    # and not at the library's 2 s limit
    assert limit_us * 1e-6 <= dt < 0.5, dt
    # the report cleared the error word; the context is usable
    assert N.lib().tvq_device_error(None) == N.TVQ_OK
    assert _gemm_bit_exact(2)
    torch.cuda.synchronize()

