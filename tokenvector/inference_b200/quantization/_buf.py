"""Buffer plumbing shared by the tv.quantization mirror.

Host buffers are numpy arrays (the reference's lists); device buffers are
torch CUDA tensors.  Only pointers and sizes cross the C ABI.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

try:  # torch is plumbing for device memory and streams only
    import torch
except Exception:  # pragma: no cover
    torch = None


def is_dev(x) -> bool:
    return torch is not None and isinstance(x, torch.Tensor) and x.is_cuda


def ptr(x):
    if x is None:
        return None
    if is_dev(x):
        assert x.is_contiguous(), "device buffers must be contiguous"
        return C.c_void_p(x.data_ptr())
    assert isinstance(x, np.ndarray) and x.flags["C_CONTIGUOUS"], "host buffers must be contiguous numpy arrays"
    return x.ctypes.data_as(C.c_void_p)


def stream_of(x):
    if is_dev(x):
        return C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    return C.c_void_p(None)


def host_f32(x) -> np.ndarray:
    a = np.asarray(x, dtype=np.float32)
    return np.ascontiguousarray(a)


def size(x) -> int:
    if x is None:
        return 0
    if is_dev(x):
        return int(x.numel())
    return int(np.asarray(x).size)
