"""GPU parity of the HBM-bound PTQ kernels (calibration, INT8 quantize,
FP8 codec) against the CPU oracle, through the C ABI.  Bit-exact."""
import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import _native as N
from tokenvector.inference_b200.quantization import engine as E
from tokenvector.inference_b200.quantization import matmul as M
from tokenvector.inference_b200.quantization import types as T

pytestmark = pytest.mark.gpu


def _same_f32(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _data(n, seed, outliers=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    if outliers and n:
        idx = rng.choice(n, max(1, n // 1000), replace=False)
        x[idx] *= 20.0
    return x


@pytest.mark.parametrize("n", [1, 2, 5, 31, 1000, 4097, 786432])
@pytest.mark.parametrize("sym", [1, 0])
def test_calibrate_minmax(n, sym):
    x = _data(n, n, outliers=True)
    g = E.calibrate_minmax(x, sym)
    o = O.calibrate_minmax(x, sym)
    assert _same_f32(g.scale, o.scale) and g.zero_point == o.zero_point
    assert _same_f32(g.min_val, o.min_val) and _same_f32(g.max_val, o.max_val)


def test_calibrate_minmax_edges():
    for x in [np.zeros(7, np.float32), np.full(9, -3.5, np.float32), np.array([1e-12, -1e-12], np.float32),
              np.array([np.nan, 1.0, 2.0], np.float32), np.array([1.0, np.nan, -4.0], np.float32),
              np.array([np.inf, 1.0], np.float32), np.array([-np.inf], np.float32)]:
        for sym in (1, 0):
            g = E.calibrate_minmax(x, sym)
            o = O.calibrate_minmax(x, sym)
            assert _same_f32(g.scale, o.scale) or (np.isnan(g.scale) and np.isnan(o.scale)), (x, sym, g, o.scale)
            assert g.zero_point == o.zero_point, (x, sym)
    g = E.calibrate_minmax(np.zeros(0, np.float32))
    assert g.scale == 1.0 and g.zero_point == 0


def test_calibrate_eight_batches_config1():
    # scale over 8 seeded [1024,768] batches
    batches = [O.gi_noise(1024 * 768, s, 1.0) for s in range(8)]
    g = E.calibrate_minmax_batches(batches, 1)
    o = O.calibrate_minmax(np.concatenate(batches), 1)
    assert _same_f32(g.scale, o.scale)


def test_quantize_symmetric_bit_exact():
    x = _data(1 << 20, 3, outliers=True)
    x[:9] = [np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-30, -1e30, 3.0, -3.0]
    for scale in [0.0123, 1.0, 0.0, 1e-9, 3.4e38]:
        q = np.empty(x.size, np.int8)
        E.quantize_int8_symmetric(x, q, scale)
        assert np.array_equal(q, O.quantize_int8_symmetric(x, scale)), scale
    # exact ties: x * (1/scale) lands on k + 0.5
    t = (np.arange(-300, 300, dtype=np.float32) + 0.5)
    q = np.empty(t.size, np.int8)
    E.quantize_int8_symmetric(t, q, 1.0)
    assert np.array_equal(q, O.quantize_int8_symmetric(t, 1.0))
    # unaligned / odd sizes and the list[i32] destination
    for n in [1, 15, 17, 33]:
        xs = x[3:3 + n].copy()
        q32 = np.zeros(n, np.int32)
        E.quantize_int8_symmetric(xs, q32, 0.05)
        assert np.array_equal(q32, O.quantize_int8_symmetric(xs, 0.05).astype(np.int32))


def test_dequantize_bit_exact():
    rng = np.random.default_rng(4)
    q = rng.integers(-127, 128, 5000).astype(np.int8)
    y = np.empty(q.size, np.float32)
    E.dequantize_int8_symmetric(q, y, 0.0173)
    assert _same_f32(y, O.dequantize_int8_symmetric(q, 0.0173))
    sc = (rng.random(50) * 0.1).astype(np.float32)
    y2 = np.empty(q.size, np.float32)
    E.dequantize_int8_per_channel(q, y2, 50, 100, sc)
    assert _same_f32(y2, O.dequantize_int8_per_channel(q, 50, 100, sc))


# cols 1025..8192 (multiple of 4) take the block-per-row kernel (row held in
# registers), the others the warp-per-row kernel
@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (64, 768), (3072, 768), (100, 1001), (64, 1600), (5, 4100),
                                       (7, 6400), (3, 8192), (2, 8196), (9, 1030)])
def test_per_channel_calibrate_and_quantize(rows, cols):
    w = (O.gi_noise(rows * cols, rows + cols) if rows * cols > 1 else np.array([0.5], np.float32)).reshape(rows, cols)
    ps = E.calibrate_per_channel_minmax(w, rows, cols)
    os_ = O.per_channel_scales(w, rows, cols)
    assert _same_f32([p.scale for p in ps], os_)
    q = np.empty(rows * cols, np.int8)
    E.quantize_int8_per_channel(w, q, rows, cols, os_)
    assert np.array_equal(q.reshape(rows, cols), O.quantize_int8_per_channel(w, rows, cols, os_))


def test_per_channel_edges():
    w = np.array([[0.0, 0.0, 0.0], [np.nan, 1.0, 2.0], [1.0, np.nan, -2.0], [1e-12, 2e-12, 0.0]], np.float32)
    ps = E.calibrate_per_channel_minmax(w, 4, 3)
    os_ = O.per_channel_scales(w, 4, 3)
    g = np.array([p.scale for p in ps], np.float32)
    assert np.array_equal(np.isnan(g), np.isnan(os_))
    assert _same_f32(g[~np.isnan(g)], os_[~np.isnan(os_)])


def _qp_fields(ps):
    return (np.array([p.scale for p in ps], np.float32), np.array([p.zero_point for p in ps], np.int64),
            np.array([p.min_val for p in ps], np.float32), np.array([p.max_val for p in ps], np.float32))


def _same_bits_nan(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


@pytest.mark.parametrize("symmetric", [1, 0])
def test_per_channel_quant_params_are_the_references(symmetric):
    """Every QuantParams field of calibrate_per_channel_minmax (engine.tkv:
    202-213 -> calibrate_minmax per row, :13-36), one launch on the GPU,
    against the oracle: scale, zero point and the row's own min / max, with
    the reference's first-occurrence rule for zero extremes of either sign
    and a NaN first element poisoning the row."""
    rng = np.random.default_rng(11 + symmetric)
    w = (rng.standard_normal((300, 77)) * 0.02).astype(np.float32)
    w[1] = 0.0
    w[2, :3] = [1.0, 0.0, -0.0]           # min 0: the +0 comes first
    w[2, 3:] = 0.5
    w[3, :3] = [1.0, -0.0, 0.0]           # min 0: the -0 comes first
    w[3, 3:] = 0.5
    w[4, :3] = [-1.0, -0.0, 0.0]          # max 0: the -0 comes first
    w[4, 3:] = -0.5
    w[5, 0] = np.nan                      # poisoned row
    w[6, 10] = np.nan                     # a NaN that never wins
    w[7] = 3.25                           # constant row (asymmetric: mx = mn + 1e-8)
    w[8] = 1e-12                          # below the 1e-8 floor
    w[9, 40] = np.inf
    ps = E.calibrate_per_channel_minmax(w, 300, 77, symmetric)
    ref = O.calibrate_per_channel_minmax(w, 300, 77, symmetric)
    gs, gz, gmn, gmx = _qp_fields(ps)
    rs = np.array([q.scale for q in ref], np.float32)
    rz = np.array([q.zero_point for q in ref], np.int64)
    rmn = np.array([q.min_val for q in ref], np.float32)
    rmx = np.array([q.max_val for q in ref], np.float32)
    assert _same_bits_nan(gs, rs) and np.array_equal(gz, rz)
    assert _same_bits_nan(gmn, rmn) and _same_bits_nan(gmx, rmx)
    if symmetric:  # the true row max, not fl32(scale) * 127
        assert gmx[0] == np.float32(np.abs(w[0]).max())


@pytest.mark.parametrize("rows,cols", [(512, 300), (40, 6400)])
def test_dynamic_rowwise(rows, cols):
    x = _data(rows * cols, 5, outliers=True).reshape(rows, cols)
    x[7, :] = 0.0
    x[9, 3] = np.nan
    q = np.empty(x.size, np.int8)
    sc = np.empty(rows, np.float32)
    E.quantize_dynamic_int8_rowwise(x, q, rows, cols, sc)
    oq, osc = O.quantize_dynamic_int8_rowwise(x, rows, cols)
    assert np.array_equal(q.reshape(rows, cols), oq)
    assert _same_f32(sc, osc)


def test_fp8_decode_all_bytes():
    b = np.arange(256, dtype=np.uint8)
    y = np.empty(256, np.float32)
    M.dequantize_fp8_e4m3(b, y)
    o = O.dequantize_fp8_e4m3(b)
    assert _same_f32(y, o)
    assert T.native_fp8_e4m3_decode(0x7E) == 448.0
    assert T.fp8e4m3_from_float(1.0).value == 0x38


def test_fp8_encode_reference_quirks_and_random():
    special = np.array([0.0, -0.0, 0.5, 1.0, -1.0, 2.5, 16.0, 240.0, 247.0, 248.0, 255.9, 256.0, 300.0, 448.0,
                        1e9, -1e9, 2.0 ** -6, 7.6 * 2.0 ** -9, 2.0 ** -9, 2.0 ** -10, 1.5 * 2.0 ** -10,
                        2.0 ** -149, -2.0 ** -149, np.nan, np.inf, -np.inf], np.float32)
    rng = np.random.default_rng(6)
    bits = rng.integers(0, 2 ** 32, 1 << 18, dtype=np.uint64).astype(np.uint32)
    rand = bits.view(np.float32)
    near = (rng.standard_normal(1 << 18) * rng.choice([1e-3, 0.05, 1, 30, 250], 1 << 18)).astype(np.float32)
    x = np.concatenate([special, rand, near])
    for xs in (x, x[: x.size - x.size % 4]):  # scalar and 4-wide vector kernels
        q = np.empty(xs.size, np.uint8)
        M.quantize_fp8_e4m3(xs, q)
        assert np.array_equal(q, O.quantize_fp8_e4m3(xs))
    # list[i32] form stores byte - 128 (matmul.tkv:65)
    q32 = np.empty(special.size, np.int32)
    M.quantize_fp8_e4m3(special, q32)
    assert np.array_equal(q32, O.quantize_fp8_e4m3(special).astype(np.int32) - 128)


@pytest.mark.parametrize("cols", [1024, 1001])
def test_fp8_scaled_quantize(cols):
    x = _data(64 * cols, 8, outliers=True).reshape(64, cols)
    amax_rows = np.abs(x).max(axis=1)
    sc = (amax_rows / 448.0).astype(np.float32)
    g = M.quantize_fp8_e4m3_scaled(x, 64, cols, sc, True)
    assert np.array_equal(g, O.quantize_fp8_e4m3_scaled(x, sc, True))
    st = np.array([np.abs(x).max() / 448.0], np.float32)
    g = M.quantize_fp8_e4m3_scaled(x, 64, cols, st, False)
    assert np.array_equal(g, O.quantize_fp8_e4m3_scaled(x, st, False))


def test_fp8_encode_all_binary32_inputs():
    """The device encoder (hardware RN-satfinite conversion where it agrees
    with the reference, the integer form elsewhere) against the oracle's
    restatement of native_fp8_e4m3_encode (types.tkv:154-191) on every one
    of the 2^32 binary32 bit patterns, in chunks of 2^26 through the device
    entry point (flat, unscaled: 16-byte loads, the vector kernel)."""
    import torch
    dev = torch.device("cuda", 0)
    st = torch.cuda.current_stream()
    chunk = 1 << 26
    xd = torch.empty(chunk, dtype=torch.float32, device=dev)
    qd = torch.empty(chunk, dtype=torch.uint8, device=dev)
    bad = 0
    for c in range(1 << 6):
        bits = np.arange(c * chunk, (c + 1) * chunk, dtype=np.uint64).astype(np.uint32)
        x = bits.view(np.float32)
        xd.copy_(torch.from_numpy(x))
        N.call("tvq_dev_quantize_fp8", xd.data_ptr(), qd.data_ptr(), 1, chunk, None, 0, N.FP8_REF, st.cuda_stream)
        bad += int((qd.cpu().numpy() != O.quantize_fp8_e4m3(x)).sum())
    assert bad == 0
