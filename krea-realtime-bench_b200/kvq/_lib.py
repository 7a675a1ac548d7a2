"""ctypes binding of libkvq.so, the C ABI declared in include/kvq.h.

The library is built in-tree (kvq/build.py) and loaded from
krea-realtime-bench_b200/libkvq.so. There is no fallback: if the library is
missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

KVQ_OK = 0
KVQ_ERR_ARG = -1
KVQ_ERR_UNSUPPORTED = -2
KVQ_ERR_CUDA = -3
KVQ_ERR_ALIGN = -4
KVQ_ERR_DEVICE = -5

# every symbol include/kvq.h declares, with (restype, argtypes)
_p, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
SIGNATURES = {
    "kvq_abi_version": (_i32, []),
    "kvq_last_error": (ctypes.c_char_p, []),
    "kvq_quantize": (_i32, [_p, _i64, _p, _p, _p, _i64, _i64, _i32, _i32, _p, _i32, _i32, _p]),
    "kvq_dequantize": (_i32, [_p, _p, _p, _i64, _p, _i64, _i64, _i32, _i32, _p, _i32, _i32, _p]),
    "kvq_requantize": (_i32, [_p, _p, _p, _i64, _p, _p, _p, _i64, _i64, _i32, _i32, _p, _i32, _i32, _p]),
    "kvq_attention": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _i32, _i64,
                             _i32, _i32, _p, _i32, _i32, _i32, _f32, _p, _i64, _p]),
    "kvq_attention_workspace_bytes": (_i32, [_i32, _i64, _i32, _i64, ctypes.POINTER(_i64)]),
    "kvq_attention_noalloc": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _i32,
                                     _i64, _i32, _i32, _p, _i32, _i32, _i32, _f32, _p]),
    "kvq_attention_stats": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _p, _i32,
                                   _i64, _i32, _i32, _p, _i32, _i32, _i32, _f32, _p]),
    "kvq_rope_quantize": (_i32, [_p, _i64, _p, _p, _p, _i64, _i64, _i32, _i32, _p, _i32, _i32, _p, _i32, _p, _p]),
    "kvq_rebuild_layers": (_i32, [_i32, _p, _i64, _p, _p, _p, _i64, _i64, _i32, _i32, _p, _i32, _i32, _p]),
    "kvq_attention_gather": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i32, _i32, _i32,
                                    _i64, _i32, _i64, _i32, _i32, _p, _i32, _i32, _i32, _f32, _p, _i64, _p]),
    "kvq_gather_barrier": (_i32, [_p, _i32, _i32, ctypes.c_uint, _i64, _p]),
    "kvq_ipc_export": (_i32, [_p, _p, ctypes.POINTER(_i64)]),
    "kvq_ipc_import": (_i32, [_p, _i64, ctypes.POINTER(_p), ctypes.POINTER(_p)]),
    "kvq_ipc_close": (_i32, [_p]),
    "kvq_test_attention_timeout": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _i32,
                                          _i64, _i32, _i32, _p, _i32, _i32, _i32, _f32, _i32, _i64, _p]),
    "kvq_device_status": (_i32, [_i32]),
}
ABI_VERSION = 3
IPC_HANDLE_BYTES = 64

_lib = None
_lock = threading.Lock()


class KVQError(RuntimeError):
    """A libkvq call returned a negative status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[kvq status {status}] {message}")
        self.status = status


def library_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = False):
    """Loads (once) and returns the ctypes handle of libkvq.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB
        if not os.path.exists(path):
            if not build_if_missing:
                raise RuntimeError(
                    f"libkvq.so not found at {path}; build it with "
                    "`python -m kvq.build` from krea-realtime-bench_b200/ (no CPU fallback exists)")
            _build.build()
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        v = lib.kvq_abi_version()
        if v != ABI_VERSION:
            raise RuntimeError(f"libkvq ABI version {v}, expected {ABI_VERSION}; rebuild the library")
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status == KVQ_OK:
        return
    msg = load().kvq_last_error().decode(errors="replace")
    if status in (KVQ_ERR_ARG, KVQ_ERR_ALIGN, KVQ_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg} [kvq status {status}]")
    raise KVQError(status, f"{what}: {msg}")
