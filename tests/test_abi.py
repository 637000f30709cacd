"""The C ABI boundary: libtvq.so loads without a GPU and exports exactly what
include/*.h declares (no compute calls here)."""
import ctypes
import os
import re

import pytest

from tokenvector.inference_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"^\s*(?:TVQ_API\s+)?(?:int|float|void|int64_t)\s+\**(tvq_\w+)\s*\(", src, flags=re.M))
    return names


def test_library_builds_and_loads():
    from tokenvector.inference_b200 import build
    build.build()
    assert os.path.exists(N.LIB_PATH)
    N.lib()


def test_every_declared_symbol_is_exported():
    decl = _declared()
    assert len(decl) >= 30
    lib = ctypes.CDLL(N.LIB_PATH)
    missing = [s for s in sorted(decl) if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    decl = _declared()
    assert decl == set(N.SIGNATURES), sorted(decl ^ set(N.SIGNATURES))


def test_version_and_error_string():
    assert N.lib().tvq_version() >= 10000
    buf = ctypes.create_string_buffer(64)
    assert N.lib().tvq_last_error(buf, 64) == 0
    assert N.lib().tvq_last_error(None, 0) == N.TVQ_ERR_INVALID


def test_argument_errors_need_no_gpu():
    # size checks come before any device work, as the reference's ValueErrors
    import numpy as np
    from tokenvector.inference_b200.quantization import matmul as M, engine as E
    with pytest.raises(ValueError):
        M.matmul_int8_per_channel(np.zeros(8, np.int8), np.zeros(12, np.int8), [], np.zeros(6, np.float32),
                                  2, 3, 4, 1.0, np.ones(2, np.float32))
    with pytest.raises(ValueError):
        E.quantize_int8_symmetric(np.zeros(4, np.float32), np.zeros(3, np.int8), 1.0)
    with pytest.raises(ValueError):
        E.calibrate_per_channel_minmax(np.zeros(4, np.float32), 0, 4)
    with pytest.raises(ValueError):
        E.quantize_int8_per_channel(np.zeros(8, np.float32), np.zeros(8, np.int8), 2, 4, np.ones(1, np.float32))


def test_attention_entry_points_refuse_bad_layouts_before_any_device_work():
    """Negative segment offsets, head counts that do not divide d and head
    dims without a kernel are refused on the host, before any copy or launch
    (so no GPU is needed to see it).  The pointers are never dereferenced."""
    import numpy as np
    fake = ctypes.c_void_p(256)  # a non-null address that must not be touched
    neg = np.array([-64, 100], np.int64)
    ok = np.array([0, 100], np.int64)
    sp = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    L = N.lib()
    # tvq_dev_attention_noalloc (fixed device scratch)
    assert L.tvq_dev_attention_noalloc(fake, sp(neg), 1, 768, 12, fake, None, None, None, None) == N.TVQ_ERR_INVALID
    assert L.tvq_dev_attention_noalloc(fake, sp(ok), 1, 768, 7, fake, None, None, None, None) == N.TVQ_ERR_INVALID
    assert L.tvq_dev_attention_noalloc(fake, sp(ok), 1, 768, 0, fake, None, None, None, None) == N.TVQ_ERR_INVALID
    assert L.tvq_dev_attention_noalloc(fake, sp(ok), 1, 8, 16, fake, None, None, None, None) == N.TVQ_ERR_INVALID
    assert L.tvq_dev_attention_noalloc(fake, sp(ok), 1, 1024, 8, fake, None, None, None,
                                       None) == N.TVQ_ERR_UNSUPPORTED  # head dim 128
    assert L.tvq_dev_attention_noalloc(fake, sp(ok), 1, (1 << 32) + 12, 12, fake, None, None, None,
                                       None) == N.TVQ_ERR_INVALID  # no narrowing to int
    # tvq_dev_attention (caller-provided scratch)
    assert L.tvq_dev_attention(fake, sp(neg), 1, 768, 12, fake, 64, fake, None, None, None,
                               None) == N.TVQ_ERR_INVALID
    assert L.tvq_dev_attention(fake, sp(ok), 1, 768, 7, fake, 64, fake, None, None, None, None) == N.TVQ_ERR_INVALID


def test_wait_selftest_rejects_out_of_range_limits_without_a_gpu():
    for bad in (0, -5, 2_000_000):
        assert N.lib().tvq_selftest_wait_timeout(bad, None) == N.TVQ_ERR_INVALID
