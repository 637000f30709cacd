"""tvq_dev_attention_noalloc: the attention entry point for callers that
cannot allocate device memory when they call (a host whose device memory
belongs to its own fixed pool, a serving loop that must not allocate because
an allocation can synchronise the device).  Its query-tile scratch is a fixed
device array inside libtvq, so this test checks, on two calls in a row with
different inputs, that it matches the allocating entry point
tvq_dev_attention: within the attention tolerance used by the other tests
(rtol 1e-4, atol 2e-6) at head dim 64, where the allocating entry point takes
the tensor-core kernel, and bit for bit at head dim 32, where both run the
same fp32 kernel; that its int8 output and amax match too; that one small
case agrees with the CPU oracle; and that a call needing more scratch than the
array holds is refused.  It lives in a file of its own that pytest collects
last and must pass in a fresh process as well as after the other tests."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from tokenvector.inference_b200 import _native as N

pytestmark = pytest.mark.gpu


def _run_both(lengths, d, heads, seed, quant=False):
    import torch
    dev = torch.device("cuda:0")
    seg = np.zeros(len(lengths) + 1, np.int64)
    seg[1:] = np.cumsum(lengths)
    T = int(seg[-1])
    qkv_h = np.random.default_rng(seed).standard_normal((T, 3 * d)).astype(np.float32)
    qkv = torch.from_numpy(qkv_h).to(dev)
    ref = torch.empty((T, d), dtype=torch.float32, device=dev)
    got = torch.full((T, d), float("nan"), dtype=torch.float32, device=dev)
    tiles = torch.empty((T + 64 * len(lengths)) * 4, dtype=torch.int32, device=dev)
    p = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    qs = torch.tensor([0.01], dtype=torch.float32, device=dev) if quant else None
    rq = torch.zeros((T, d), dtype=torch.int8, device=dev) if quant else None
    gq = torch.zeros((T, d), dtype=torch.int8, device=dev) if quant else None
    ra = torch.zeros(1, dtype=torch.int32, device=dev) if quant else None
    ga = torch.zeros(1, dtype=torch.int32, device=dev) if quant else None
    sp = seg.ctypes.data_as(C.c_void_p)
    N.call("tvq_dev_attention", p(qkv), sp, len(lengths), d, heads, p(tiles), T + 64 * len(lengths), p(ref),
           p(rq), p(qs), p(ra), None)
    N.call("tvq_dev_attention_noalloc", p(qkv), sp, len(lengths), d, heads, p(got), p(gq), p(qs), p(ga), None)
    torch.cuda.synchronize()
    out = {"got": got.cpu().numpy(), "ref": ref.cpu().numpy(), "qkv": qkv_h, "seg": seg}
    if quant:
        out.update(gq=gq.cpu().numpy(), rq=rq.cpu().numpy(), ga=ga.cpu().numpy().view(np.float32)[0],
                   ra=ra.cpu().numpy().view(np.float32)[0])
    return out


def test_noalloc_attention_matches_allocating_entry_point_twice():
    r1 = _run_both([300, 77, 1], 768, 12, seed=1)
    assert np.allclose(r1["got"], r1["ref"], rtol=1e-4, atol=2e-6)
    # second call reuses the same scratch with a different layout
    r2 = _run_both([1024, 64], 128, 2, seed=2)
    assert np.allclose(r2["got"], r2["ref"], rtol=1e-4, atol=2e-6)


def test_noalloc_attention_same_bits_where_both_run_the_fp32_kernel():
    # head dim 32: both entry points run the fp32 SIMT kernel on the same
    # tiles, so every output, int8 value and the amax are identical
    for lengths, seed in (([200, 65, 3], 3), ([130], 4)):
        r = _run_both(lengths, 128, 4, seed=seed, quant=True)
        assert np.array_equal(r["got"].view(np.uint32), r["ref"].view(np.uint32))
        assert np.array_equal(r["gq"], r["rq"])
        assert r["ga"] == r["ra"] and r["ga"] == np.abs(r["got"]).max()


def test_noalloc_attention_matches_the_oracle():
    r = _run_both([70, 33], 128, 2, seed=5)
    want = O.attention_causal(r["qkv"], 2, r["seg"])
    assert np.allclose(r["got"], want, rtol=1e-4, atol=2e-6)


def test_noalloc_attention_rejects_oversized_call():
    import torch
    seg = np.array([0, 32768 * 64 + 1], np.int64)  # 32769 tiles
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda:0")
    with pytest.raises(ValueError, match="no-allocation scratch"):
        N.call("tvq_dev_attention_noalloc", C.c_void_p(dummy.data_ptr()), seg.ctypes.data_as(C.c_void_p), 1, 64, 4,
               C.c_void_p(dummy.data_ptr()), None, None, None, None)
