"""PTQ artefacts (tokenvector/inference_b200/ptq.py): the calibrated INT8
linears on disk, reloaded bit for bit (f32 as IEEE bits, as the reference's
checkpoints keep them, tv/training/trainer.tkv:857-958), integrity-checked.
No GPU needed."""
import numpy as np
import pytest

from tokenvector.inference_b200 import ptq


def _linears(seed=0):
    rng = np.random.default_rng(seed)
    out = []
    for i, (n, k) in enumerate([(96, 64), (64, 96), (7, 33)]):
        sw = (rng.random(n) * 1e-3).astype(np.float32)
        sw[0] = np.float32(1e-45)           # a subnormal scale survives
        bias = rng.standard_normal(n).astype(np.float32)
        bias[1] = -0.0                      # signed zero survives
        bias[2] = np.frombuffer(np.uint32(0x7FC00123).tobytes(), np.float32)[0]  # NaN payload survives
        out.append(ptq.QuantLinear("blk.%d" % i, rng.integers(-127, 128, (n, k)).astype(np.int8), scales_w=sw,
                                   bias=bias, scale_a=float(rng.random()) * 0.05, act=6 if i == 1 else 0))
    out.append(ptq.QuantLinear("per_tensor", rng.integers(-127, 128, (16, 32)).astype(np.int8), scale_b=0.0123,
                               scale_a=0.5))
    return out


def test_round_trip_is_bit_exact(tmp_path):
    lins = _linears()
    p = str(tmp_path / "m.tvqptq")
    ptq.save(p, lins, meta={"model": "test"})
    back, meta = ptq.load(p)
    assert meta == {"model": "test"}
    assert len(back) == len(lins)
    for a, b in zip(lins, back):
        assert a == b, a.name
    assert back[0].bias.view(np.uint32)[1] == 0x80000000
    assert back[0].bias.view(np.uint32)[2] == 0x7FC00123


def test_corruption_is_detected(tmp_path):
    p = str(tmp_path / "m.tvqptq")
    ptq.save(p, _linears(1))
    raw = bytearray(open(p, "rb").read())
    bad = bytearray(raw)
    bad[-70] ^= 0x01  # a payload byte
    open(p, "wb").write(bytes(bad))
    with pytest.raises(ValueError, match="CRC"):
        ptq.load(p)
    open(p, "wb").write(bytes(raw[:-200]))
    with pytest.raises(ValueError, match="truncated"):
        ptq.load(p)
    open(p, "wb").write(b"NOTPTQ!\n" + bytes(raw[8:]))
    with pytest.raises(ValueError, match="not a TVQPTQ1"):
        ptq.load(p)


def test_quant_linear_checks_like_the_reference():
    w = np.zeros((4, 8), np.int8)
    with pytest.raises(ValueError, match="scales_w smaller than N"):  # matmul.tkv:18-19
        ptq.QuantLinear("x", w, scales_w=np.ones(3, np.float32))
    with pytest.raises(ValueError, match="exactly one"):
        ptq.QuantLinear("x", w)
    with pytest.raises(ValueError, match="duplicate"):
        ptq.save("/dev/null", [ptq.QuantLinear("x", w, scale_b=1.0), ptq.QuantLinear("x", w, scale_b=1.0)])
