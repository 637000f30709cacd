"""tvq_dev_attention_noalloc: the attention entry point for callers that
cannot allocate device memory (a host whose device memory belongs to its own
pool, a serving loop that must not allocate).  Its query-tile scratch is a
fixed device array inside libtvq, so this test checks that two calls in a
row, with different inputs, match the allocating entry point
tvq_dev_attention within the attention tolerance used by the other tests
(rtol 1e-4, atol 2e-6), and that a call needing more scratch than the array
holds is refused.  It lives in a file of its own that pytest collects last
and must pass in a fresh process as well as after the other tests."""
import ctypes as C

import numpy as np
import pytest

from tokenvector.inference_b200 import _native as N

pytestmark = pytest.mark.gpu


def _run_both(lengths, d, heads, seed):
    import torch
    dev = torch.device("cuda:0")
    seg = np.zeros(len(lengths) + 1, np.int64)
    seg[1:] = np.cumsum(lengths)
    T = int(seg[-1])
    qkv = torch.from_numpy(np.random.default_rng(seed).standard_normal((T, 3 * d)).astype(np.float32)).to(dev)
    ref = torch.empty((T, d), dtype=torch.float32, device=dev)
    got = torch.full((T, d), float("nan"), dtype=torch.float32, device=dev)
    tiles = torch.empty((T + 64 * len(lengths)) * 4, dtype=torch.int32, device=dev)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    sp = seg.ctypes.data_as(C.c_void_p)
    N.call("tvq_dev_attention", p(qkv), sp, len(lengths), d, heads, p(tiles), T + 64 * len(lengths), p(ref),
           None, None, None, None)
    N.call("tvq_dev_attention_noalloc", p(qkv), sp, len(lengths), d, heads, p(got), None, None, None, None)
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy()


def test_noalloc_attention_matches_allocating_entry_point_twice():
    got1, ref1 = _run_both([300, 77, 1], 768, 12, seed=1)
    assert np.allclose(got1, ref1, rtol=1e-4, atol=2e-6)
    # second call reuses the same scratch with a different layout
    got2, ref2 = _run_both([1024, 64], 128, 2, seed=2)
    assert np.allclose(got2, ref2, rtol=1e-4, atol=2e-6)


def test_noalloc_attention_rejects_oversized_call():
    import torch
    seg = np.array([0, 32768 * 64 + 1], np.int64)  # 32769 tiles
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda:0")
    with pytest.raises(ValueError, match="no-allocation scratch"):
        N.call("tvq_dev_attention_noalloc", C.c_void_p(dummy.data_ptr()), seg.ctypes.data_as(C.c_void_p), 1, 64, 4,
               C.c_void_p(dummy.data_ptr()), None, None, None, None)
