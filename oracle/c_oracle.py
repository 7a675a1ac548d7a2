"""ctypes binding of the C oracle (oracle/kvq_oracle.c); test infrastructure only.

Loads oracle/_build/libkvq_oracle.so, building it with `make -C oracle` when it
is missing. All arrays are numpy; bf16 values travel as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libkvq_oracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        L = ctypes.CDLL(_SO)
        p = ctypes.c_void_p
        i64, i32 = ctypes.c_int64, ctypes.c_int
        L.kvqo_quantize.argtypes = [p, i64, p, p, i64, i32, i32, p, i32, i32, i32]
        L.kvqo_quantize.restype = i32
        L.kvqo_dequantize.argtypes = [p, p, p, i64, i32, i32, p, i32, i32, i32]
        L.kvqo_dequantize.restype = i32
        L.kvqo_check_fast_codes.argtypes = [i32, ctypes.c_float, i32,
                                            ctypes.POINTER(ctypes.c_uint32)]
        L.kvqo_check_fast_codes.restype = ctypes.c_longlong
        L.kvqo_check_fast_codes_rcp.argtypes = [i32, ctypes.c_float, i32, i32,
                                                ctypes.POINTER(ctypes.c_uint32)]
        L.kvqo_check_fast_codes_rcp.restype = ctypes.c_longlong
        L.kvqo_check_scale_div.argtypes = [i32]
        L.kvqo_check_scale_div.restype = ctypes.c_longlong
        _lib = L
    return _lib


def _edges(bands) -> np.ndarray:
    return np.ascontiguousarray(np.array(bands, dtype=np.int32).reshape(-1))


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def quantize(x_bits: np.ndarray, bands, bits: int = 4, threads: int | None = None):
    """[L, H, D] bf16 bits (token-strided allowed) -> (codes, scales bf16 bits)."""
    x = np.asarray(x_bits)
    assert x.dtype == np.uint16 and x.ndim == 3
    L, H, D = x.shape
    if x.strides[1] != D * 2 or x.strides[2] != 2:
        x = np.ascontiguousarray(x)
    row_stride = x.strides[0] // 2
    G = len(bands)
    codes = np.empty((L, H, D // 2 if bits == 4 else D), np.uint8)
    scales = np.empty((L, H, G), np.uint16)
    e = _edges(bands)
    rc = lib().kvqo_quantize(_ptr(x), row_stride, _ptr(codes), _ptr(scales), L, H, D,
                             _ptr(e), G, bits, threads or os.cpu_count() or 1)
    if rc != 0:
        raise ValueError("kvqo_quantize rejected its arguments")
    return codes, scales


def dequantize(codes: np.ndarray, scales_bits: np.ndarray, bands, head_dim: int,
               bits: int = 4, threads: int | None = None) -> np.ndarray:
    c = np.ascontiguousarray(codes)
    s = np.ascontiguousarray(scales_bits)
    L, H = c.shape[:2]
    out = np.empty((L, H, head_dim), np.uint16)
    e = _edges(bands)
    rc = lib().kvqo_dequantize(_ptr(c), _ptr(s), _ptr(out), L, H, head_dim, _ptr(e),
                               len(bands), bits, threads or os.cpu_count() or 1)
    if rc != 0:
        raise ValueError("kvqo_dequantize rejected its arguments")
    return out


def check_fast_codes(qmax: int, exact_below: float, threads: int | None = None):
    """Exhaustive count of (x, amax) pairs where the kernel's division-free code
    formula differs from the reference's divide; returns (count, first_pair)."""
    first = ctypes.c_uint32()
    n = lib().kvqo_check_fast_codes(qmax, exact_below, threads or os.cpu_count() or 1,
                                    ctypes.byref(first))
    return int(n), (first.value >> 16, first.value & 0xFFFF)


def check_fast_codes_any_rcp(qmax: int, exact_below: float, threads: int | None = None):
    """As check_fast_codes, but the formula must hold for every reciprocal within
    one ulp of 1/s."""
    first = ctypes.c_uint32()
    n = lib().kvqo_check_fast_codes_rcp(qmax, exact_below, 1, threads or os.cpu_count() or 1,
                                        ctypes.byref(first))
    return int(n), (first.value >> 16, first.value & 0xFFFF)


def check_scale_div(qmax: int) -> int:
    """Exhaustive count of bf16 amax where the kernel's divide-free group scale
    differs from the IEEE quotient amax / qmax."""
    return int(lib().kvqo_check_scale_div(qmax))
