"""GPU calibration methods (calibrate_kl / _percentile / _mse,
tv/quantization/engine.tkv:42-197) against the oracle on the same data:
percentile bit-exact (exact radix select); KL bit-exact (the same binary64
loops in the same order; log() of CUDA and of the host C library may differ
in the last bit, so a differing threshold must be a near tie of the KL
values); MSE the same candidate, or one whose error is within 1e-12 relative
of the oracle's minimum (the device sums in another order)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import _native as N

pytestmark = pytest.mark.gpu


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _call(name, x, *args):
    s = C.c_float(0)
    z = C.c_int64(0)
    lo = C.c_float(0)
    hi = C.c_float(0)
    N.call(name, _p(x), x.size, *args, C.byref(s), C.byref(z), C.byref(lo), C.byref(hi))
    return s.value, z.value, lo.value, hi.value


def _data(n, seed, outliers=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    if outliers:
        x[rng.choice(n, max(n // 1000, 1), replace=False)] *= 20
    return x


CASES = [(1, 0), (7, 1), (1000, 2), (786432, 3), (3_000_001, 4)]


@pytest.mark.parametrize("n,seed", CASES)
@pytest.mark.parametrize("pct,sym", [(99.99, 1), (99.0, 0), (50.0, 1), (100.0, 0)])
def test_calibrate_percentile_bit_exact(n, seed, pct, sym):
    x = _data(n, seed)
    got = _call("tvq_calibrate_percentile", x, pct, sym)
    r = O.calibrate_percentile(x, pct, sym)
    assert got == (r.scale, r.zero_point, r.min_val, r.max_val)


def test_calibrate_percentile_errors_and_empty():
    x = _data(10, 0)
    with pytest.raises(ValueError):
        _call("tvq_calibrate_percentile", x, 0.0, 1)
    e = np.zeros(0, np.float32)
    assert _call("tvq_calibrate_percentile", e, 0.0, 1)[0] == 1.0  # empty: identity before the range check


@pytest.mark.parametrize("n,seed", CASES)
def test_calibrate_kl_matches_oracle(n, seed):
    x = _data(n, seed)
    got = _call("tvq_calibrate_kl", x, 2048, 128)
    r = O.calibrate_kl(x)
    assert got == (r.scale, r.zero_point, r.min_val, r.max_val)


def test_calibrate_kl_other_bins_and_tiny():
    x = _data(100000, 9)
    for nb, tb in ((1024, 64), (4096, 128), (512, 512)):
        got = _call("tvq_calibrate_kl", x, nb, tb)
        r = O.calibrate_kl(x, nb, tb)
        assert got == (r.scale, r.zero_point, r.min_val, r.max_val)
    t = np.array([1e-9, -3e-9, 0.0], np.float32)  # max |x| < 1e-8 -> calibrate_minmax(data, 1)
    r = O.calibrate_minmax(t, 1)
    assert _call("tvq_calibrate_kl", t, 2048, 128) == (r.scale, r.zero_point, r.min_val, r.max_val)


@pytest.mark.parametrize("n,seed", CASES[:4])
def test_calibrate_mse_matches_oracle(n, seed):
    x = _data(n, seed)
    got = _call("tvq_calibrate_mse", x, 50)
    r = O.calibrate_mse(x)
    if got != (r.scale, r.zero_point, r.min_val, r.max_val):
        curve = O.calibrate_mse_curve(x)
        am = float(np.abs(x).max())
        c = int(round(got[3] / (am / 50)))
        assert abs(curve[c - 1] - curve.min()) <= 1e-12 * curve.min()


def test_calibrate_mse_curve_device_form():
    import torch
    x = _data(200000, 5)
    tx = torch.from_numpy(x).cuda()
    curve = torch.zeros(50, dtype=torch.float64, device="cuda")
    out4 = torch.zeros(4, dtype=torch.float32, device="cuda")
    fb = C.c_int(0)
    N.call("tvq_dev_calibrate_mse_curve", C.c_void_p(tx.data_ptr()), x.size, 50, C.c_void_p(curve.data_ptr()),
           C.c_void_p(out4.data_ptr()), C.byref(fb), None)
    torch.cuda.synchronize()
    ref = O.calibrate_mse_curve(x)
    assert fb.value == 0
    assert np.allclose(curve.cpu().numpy(), ref, rtol=1e-12, atol=0)
