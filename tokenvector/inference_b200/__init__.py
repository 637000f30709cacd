"""B200-native PTQ linear path of TokenVector.Inference.

Mirrors the reference's ``tv.quantization`` functions and its ``QuantizedGemm``
graph node on top of libtvq.so (hand-written sm_100a CUDA behind a C ABI,
declared in include/tvq.h).  There is no CPU fallback: importing a compute
entry point without the built library raises.
"""
from . import _native  # noqa: F401

__all__ = ["_native"]
