"""PTQ artefacts: the calibrated INT8 form of a set of linear layers, on disk.

The reference quantizes at run time only (tv/quantization/engine.tkv: the
calibration functions return QuantParams, quantize_int8_per_channel fills a
list) and keeps nothing: every session start recalibrates.  A PTQ artefact
holds what a QuantizedGemm node needs (session.tkv:678-697) for each linear:
the per-output-channel int8 weights W [N, K], their scales_w [N] (or one
scale_b), the bias [N] and the activation scale scale_a calibrated for its
input, so that a session can be built without recalibrating and runs the
same bits as the one that produced it.

Format (TVQPTQ1): one ASCII line "TVQPTQ1", one line of JSON (the header),
then the tensor payloads, each starting at a multiple of 64 bytes from the
end of the header line.  f32 values are stored as their IEEE binary32 bits
(little endian), so a reload is bit-exact -- the convention of the
reference's own checkpoints (tv/training/trainer.tkv:857-958, which write
f64_to_f32_bits of every value).  Every payload carries a CRC-32.

Header: {"format": "TVQPTQ1", "meta": {...}, "tensors": {name: {"dtype":
"int8"|"f32", "shape": [...], "offset": o, "nbytes": b, "crc32": c}},
"linears": [{"name", "n", "k", "w", "scales_w", "bias" (or null),
"scale_a_bits", "scale_b_bits" (per-tensor weights, else null), "act"}]}
"""
from __future__ import annotations

import json
import zlib

import numpy as np

MAGIC = b"TVQPTQ1\n"
_ALIGN = 64
_DT = {"int8": np.int8, "f32": np.float32}


def f32_bits(x: float) -> int:
    """The binary32 bit pattern of x (rounded to f32 first)."""
    return int(np.array([x], np.float32).view(np.uint32)[0])


def f32_from_bits(b: int) -> float:
    return float(np.array([b], np.uint32).view(np.float32)[0])


def _same(a, b) -> bool:
    if a is None or b is None:
        return a is None and b is None
    view = np.uint8 if a.dtype == np.int8 else np.uint32
    return a.dtype == b.dtype and a.shape == b.shape and np.array_equal(a.view(view), b.view(view))


class QuantLinear:
    """One calibrated linear: W int8 [n, k] (row = output channel), per-channel
    scales_w [n] (or scale_b for a per-tensor weight), bias [n] or None, the
    input's activation scale scale_a, and the activation the layer applies
    after its QuantizedGemm (TVQ_ACT_* code; 0 = none)."""

    def __init__(self, name: str, w, scales_w=None, bias=None, scale_a: float = 1.0, scale_b=None, act: int = 0):
        self.name = name
        self.w = np.ascontiguousarray(w, np.int8)
        if self.w.ndim != 2:
            raise ValueError("w must be [n, k]")
        self.n, self.k = self.w.shape
        self.scales_w = None if scales_w is None else np.ascontiguousarray(scales_w, np.float32).ravel()
        self.scale_b = None if scale_b is None else float(np.float32(scale_b))
        if (self.scales_w is None) == (self.scale_b is None):
            raise ValueError("exactly one of scales_w (per channel) or scale_b (per tensor)")
        if self.scales_w is not None and self.scales_w.size < self.n:
            raise ValueError("scales_w smaller than N")  # matmul.tkv:18-19
        self.bias = None if bias is None else np.ascontiguousarray(bias, np.float32).ravel()
        if self.bias is not None and self.bias.size < self.n:
            raise ValueError("bias smaller than N")
        self.scale_a = float(np.float32(scale_a))
        self.act = int(act)

    def __eq__(self, other):
        return (isinstance(other, QuantLinear) and self.name == other.name and _same(self.w, other.w)
                and _same(self.scales_w, other.scales_w) and _same(self.bias, other.bias)
                and f32_bits(self.scale_a) == f32_bits(other.scale_a)
                and (self.scale_b is None) == (other.scale_b is None)
                and (self.scale_b is None or f32_bits(self.scale_b) == f32_bits(other.scale_b))
                and self.act == other.act)


def save(path: str, linears, meta: dict | None = None) -> None:
    """Write the linears (QuantLinear) as a TVQPTQ1 artefact."""
    tensors, blobs, entries = {}, [], []
    offset = 0

    def add(name, arr, dt):
        nonlocal offset
        a = np.ascontiguousarray(arr, _DT[dt])
        raw = a.tobytes()
        tensors[name] = {"dtype": dt, "shape": list(a.shape), "offset": offset, "nbytes": len(raw),
                         "crc32": zlib.crc32(raw) & 0xFFFFFFFF}
        pad = (-len(raw)) % _ALIGN
        blobs.append(raw + b"\0" * pad)
        offset += len(raw) + pad
        return name

    names = set()
    for L in linears:
        if L.name in names:
            raise ValueError("duplicate linear name %r" % L.name)
        names.add(L.name)
        entries.append({
            "name": L.name, "n": L.n, "k": L.k,
            "w": add(L.name + ".w", L.w, "int8"),
            "scales_w": add(L.name + ".scales_w", L.scales_w, "f32") if L.scales_w is not None else None,
            "bias": add(L.name + ".bias", L.bias, "f32") if L.bias is not None else None,
            "scale_a_bits": f32_bits(L.scale_a),
            "scale_b_bits": f32_bits(L.scale_b) if L.scale_b is not None else None,
            "act": L.act,
        })
    header = {"format": "TVQPTQ1", "meta": meta or {}, "tensors": tensors, "linears": entries}
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(json.dumps(header, sort_keys=True).encode("ascii") + b"\n")
        for b in blobs:
            f.write(b)


def load(path: str):
    """Read a TVQPTQ1 artefact: (list of QuantLinear, meta dict).  Raises
    ValueError on a bad magic, a truncated payload or a CRC mismatch."""
    with open(path, "rb") as f:
        if f.read(len(MAGIC)) != MAGIC:
            raise ValueError("not a TVQPTQ1 artefact")
        header = json.loads(f.readline().decode("ascii"))
        body = f.read()
    if header.get("format") != "TVQPTQ1":
        raise ValueError("unknown artefact format")
    arrays = {}
    for name, t in header["tensors"].items():
        raw = body[t["offset"]:t["offset"] + t["nbytes"]]
        if len(raw) != t["nbytes"]:
            raise ValueError("truncated payload %r" % name)
        if zlib.crc32(raw) & 0xFFFFFFFF != t["crc32"]:
            raise ValueError("CRC mismatch in %r" % name)
        arrays[name] = np.frombuffer(raw, dtype=_DT[t["dtype"]]).reshape(t["shape"]).copy()
    out = []
    for e in header["linears"]:
        out.append(QuantLinear(
            e["name"], arrays[e["w"]],
            scales_w=arrays[e["scales_w"]] if e["scales_w"] else None,
            bias=arrays[e["bias"]] if e["bias"] else None,
            scale_a=f32_from_bits(e["scale_a_bits"]),
            scale_b=f32_from_bits(e["scale_b_bits"]) if e["scale_b_bits"] is not None else None,
            act=e["act"]))
    return out, header["meta"]
