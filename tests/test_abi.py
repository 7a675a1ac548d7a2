"""libkvq.so loads and exports exactly the C ABI of include/kvq.h; argument
validation runs on the host (no GPU needed for these calls)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import REPO


def _declared():
    names = []
    for f in os.listdir(os.path.join(REPO, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(REPO, "include", f)).read()
            names += re.findall(r"KVQ_API\s+[\w\s\*]+?\b(kvq_\w+)\s*\(", src)
    return sorted(set(names))


def test_every_declared_symbol_is_exported(libkvq):
    from kvq import _lib
    names = _declared()
    assert "kvq_quantize" in names and "kvq_last_error" in names
    for n in names:
        assert hasattr(libkvq, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.library_path()], capture_output=True,
                         text=True).stdout
    exported = sorted(set(re.findall(r"\bT (kvq_\w+)", out)))
    assert exported == names
    assert set(_lib.SIGNATURES) == set(names)


def test_abi_version(libkvq):
    assert libkvq.kvq_abi_version() == 3


def _cb(bands=((0, 44), (44, 86), (86, 128))):
    cb = np.zeros(128, np.int32)
    for g, (lo, hi) in enumerate(bands):
        cb[lo:hi] = g
    return cb


def test_quantize_rejects_bad_arguments_without_launching(libkvq):
    cb = _cb()
    p = ctypes.c_void_p(16)
    cbp = cb.ctypes.data_as(ctypes.c_void_p)
    # bits 5
    rc = libkvq.kvq_quantize(p, 5120, p, p, None, 0, 4, 40, 128, cbp, 3, 5, None)
    assert rc == -1 and b"bits" in libkvq.kvq_last_error()
    # chan_band value out of range
    bad = cb.copy(); bad[3] = 7
    rc = libkvq.kvq_quantize(p, 5120, p, p, None, 0, 4, 40, 128, bad.ctypes.data_as(ctypes.c_void_p), 3, 4, None)
    assert rc == -1 and b"chan_band[3]" in libkvq.kvq_last_error()
    # an empty group
    rc = libkvq.kvq_quantize(p, 5120, p, p, None, 0, 4, 40, 128, cbp, 4, 4, None)
    assert rc == -1 and b"group 3" in libkvq.kvq_last_error()
    # unsupported head_dim
    rc = libkvq.kvq_quantize(p, 5120, p, p, None, 0, 4, 40, 12, cbp, 3, 4, None)
    assert rc == -2
    # misaligned x
    rc = libkvq.kvq_quantize(ctypes.c_void_p(18), 5120, p, p, None, 0, 4, 40, 128, cbp, 3, 4, None)
    assert rc == -4 and b"aligned" in libkvq.kvq_last_error()
    # token stride too small
    rc = libkvq.kvq_quantize(p, 100, p, p, None, 0, 4, 40, 128, cbp, 3, 4, None)
    assert rc == -1
    # zero tokens is a no-op success
    assert libkvq.kvq_quantize(p, 5120, p, p, None, 0, 0, 40, 128, cbp, 3, 4, None) == 0


def test_dequantize_rejects_bad_arguments_without_launching(libkvq):
    cb = _cb()
    p = ctypes.c_void_p(16)
    cbp = cb.ctypes.data_as(ctypes.c_void_p)
    rc = libkvq.kvq_dequantize(p, p, None, 0, p, 5120, 4, 40, 128, cbp, 3, 3, None)
    assert rc == -1
    rc = libkvq.kvq_dequantize(p, p, None, 0, ctypes.c_void_p(8), 5120, 4, 40, 128, cbp, 3, 4, None)
    assert rc == -4


def test_requantize_rejects_bad_arguments_without_launching(libkvq):
    cb = _cb()
    p = ctypes.c_void_p(16)
    cbp = cb.ctypes.data_as(ctypes.c_void_p)
    # int8 codes and a generic group map are not covered by the fused kernel
    assert libkvq.kvq_requantize(p, p, None, 0, p, p, None, 0, 4, 40, 128, cbp, 3, 8, None) == -2
    blind16 = np.repeat(np.arange(8, dtype=np.int32), 16)
    assert libkvq.kvq_requantize(p, p, None, 0, p, p, None, 0, 4, 40, 128,
                                 blind16.ctypes.data_as(ctypes.c_void_p), 8, 4, None) == -2
    # exact tokens without their bf16 rows, sink tokens without a sink
    assert libkvq.kvq_requantize(p, p, None, 5, p, p, None, 0, 4, 40, 128, cbp, 3, 4, None) == -1
    assert libkvq.kvq_requantize(p, p, None, 0, p, p, None, 5, 4, 40, 128, cbp, 3, 4, None) == -1
    # misaligned destination codes
    rc = libkvq.kvq_requantize(p, p, None, 0, ctypes.c_void_p(24), p, None, 0, 4, 40, 128, cbp, 3, 4, None)
    assert rc == -4 and b"aligned" in libkvq.kvq_last_error()
    # zero tokens is a no-op success
    assert libkvq.kvq_requantize(p, p, None, 0, p, p, None, 0, 0, 40, 128, cbp, 3, 4, None) == 0


def test_python_error_mapping(libkvq):
    from kvq import _lib
    cb = _cb()
    p = ctypes.c_void_p(16)
    rc = libkvq.kvq_quantize(p, 5120, p, p, None, 0, 4, 40, 128, cb.ctypes.data_as(ctypes.c_void_p), 3, 5, None)
    with pytest.raises(ValueError, match="bits"):
        _lib.check(rc, "kvq_quantize")
