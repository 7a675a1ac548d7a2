"""Torch-facing wrappers of the libkvq C ABI.

Every op validates shapes/dtypes/devices on the host, passes raw device pointers
to libkvq and launches on the current torch stream of the tensors' device. There
is no CPU path: tensors on any device other than CUDA raise.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _host_map(chan_band) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(chan_band, dtype=np.int32))
    if a.ndim != 1:
        raise ValueError("chan_band must be one-dimensional")
    return a


def _require_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"expected a torch.Tensor, got {type(t).__name__}")
        if t.device.type != "cuda":
            raise RuntimeError(
                f"kvq ops run on CUDA (sm_100) tensors only; got a tensor on {t.device} "
                "(the B200 build has no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _rows_view_ok(t: torch.Tensor, name: str, inner: int) -> int:
    """[T, H, inner] with contiguous [H, inner] block; returns the token stride."""
    if t.dim() != 3:
        raise ValueError(f"{name} must be 3-D [tokens, heads, {inner}], got {tuple(t.shape)}")
    if t.stride(2) != 1 or t.stride(1) != t.shape[2]:
        raise ValueError(f"{name} must have a contiguous [heads, channels] block per token")
    return t.stride(0)


def quantize_into(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, chan_band,
                  n_groups: int, bits: int = 4, sink: torch.Tensor | None = None,
                  sink_tokens: int = 0) -> None:
    """Quantize x [L, H, D] bf16 into codes/scales (views of any cache slice).

    Rows of x with token index < sink_tokens are also copied to sink (which
    points at the sink row of x's first token).
    """
    dev = _require_cuda(x, codes, scales, sink)
    if x.dtype != torch.bfloat16:
        raise TypeError(f"x must be bfloat16, got {x.dtype}")
    L, H, D = x.shape
    xs = _rows_view_ok(x, "x", D)
    cw = D // 2 if bits == 4 else D
    if codes.dtype != torch.uint8 or tuple(codes.shape) != (L, H, cw) or not codes.is_contiguous():
        raise ValueError(f"codes must be contiguous uint8 {(L, H, cw)}, got {codes.dtype} {tuple(codes.shape)}")
    if scales.dtype != torch.bfloat16 or tuple(scales.shape) != (L, H, n_groups) or not scales.is_contiguous():
        raise ValueError(f"scales must be contiguous bf16 {(L, H, n_groups)}")
    if sink is not None:
        ns = min(sink_tokens, L)
        if sink.dtype != torch.bfloat16 or sink.shape[0] < ns or tuple(sink.shape[1:]) != (H, D) \
                or not sink.is_contiguous():
            raise ValueError("sink must be contiguous bf16 [>=sink_tokens, H, D]")
    cb = _host_map(chan_band)
    if cb.shape[0] != D:
        raise ValueError(f"chan_band has {cb.shape[0]} entries, head_dim is {D}")
    with torch.cuda.device(dev):
        rc = _lib.load().kvq_quantize(
            _ptr(x), xs, _ptr(codes), _ptr(scales), _ptr(sink), int(sink_tokens) if sink is not None else 0,
            L, H, D, cb.ctypes.data_as(ctypes.c_void_p), int(n_groups), int(bits), _stream(dev))
    _lib.check(rc, "kvq_quantize")


def rope_quantize_into(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, chan_band, n_groups: int,
                       bits: int, freqs: torch.Tensor, positions: torch.Tensor, sink: torch.Tensor | None = None,
                       sink_tokens: int = 0) -> None:
    """quantize_into() of pre-rotary keys x [L, H, 128]: rotated in the kernel by
    freqs [P, 64, 2] float64 (kvq.rope.freqs) at positions [L, 3] int32 (frame,
    height, width; kvq.rope.grid_positions), as the upstream runtime rotates
    before its cache write (kvq_rope_quantize)."""
    dev = _require_cuda(x, codes, scales, sink, freqs, positions)
    if x.dtype != torch.bfloat16:
        raise TypeError(f"x must be bfloat16, got {x.dtype}")
    L, H, D = x.shape
    xs = _rows_view_ok(x, "x", D)
    cw = D // 2 if bits == 4 else D
    if codes.dtype != torch.uint8 or tuple(codes.shape) != (L, H, cw) or not codes.is_contiguous():
        raise ValueError(f"codes must be contiguous uint8 {(L, H, cw)}")
    if scales.dtype != torch.bfloat16 or tuple(scales.shape) != (L, H, n_groups) or not scales.is_contiguous():
        raise ValueError(f"scales must be contiguous bf16 {(L, H, n_groups)}")
    if freqs.dtype != torch.float64 or freqs.dim() != 3 or tuple(freqs.shape[1:]) != (64, 2) \
            or not freqs.is_contiguous():
        raise ValueError("freqs must be contiguous float64 [max_pos, 64, 2]")
    if positions.dtype != torch.int32 or tuple(positions.shape) != (L, 3) or not positions.is_contiguous():
        raise ValueError(f"positions must be contiguous int32 {(L, 3)}")
    if sink is not None and (sink.dtype != torch.bfloat16 or sink.shape[0] < min(sink_tokens, L)
                             or tuple(sink.shape[1:]) != (H, D) or not sink.is_contiguous()):
        raise ValueError("sink must be contiguous bf16 [>=sink_tokens, H, D]")
    cb = _host_map(chan_band)
    with torch.cuda.device(dev):
        rc = _lib.load().kvq_rope_quantize(
            _ptr(x), xs, _ptr(codes), _ptr(scales), _ptr(sink), int(sink_tokens) if sink is not None else 0,
            L, H, D, cb.ctypes.data_as(ctypes.c_void_p), int(n_groups), int(bits), _ptr(freqs), freqs.shape[0],
            _ptr(positions), _stream(dev))
    _lib.check(rc, "kvq_rope_quantize")


def quantize_layers_into(xs: list[torch.Tensor], codes: list[torch.Tensor], scales: list[torch.Tensor], chan_band,
                         n_groups: int, bits: int = 4, sinks: list[torch.Tensor | None] | None = None,
                         sink_tokens: int = 0) -> None:
    """quantize_into() of n tensors of one shape ([L, H, D] bf16 each, one token
    stride) in a single launch (kvq_rebuild_layers): the layers x {K, V} of a
    rebuild or an append. Results are bit-identical to n quantize_into() calls."""
    n = len(xs)
    if not 1 <= n <= 96 or len(codes) != n or len(scales) != n or (sinks is not None and len(sinks) != n):
        raise ValueError("1 to 96 tensors, with one codes/scales (and sink) entry each")
    dev = _require_cuda(*xs, *codes, *scales, *(sinks or []))
    L, H, D = xs[0].shape
    cw = D // 2 if bits == 4 else D
    stride = None
    for i in range(n):
        x = xs[i]
        if x.dtype != torch.bfloat16 or tuple(x.shape) != (L, H, D):
            raise ValueError(f"tensor {i}: x must be bf16 {(L, H, D)}")
        st = _rows_view_ok(x, "x", D)
        if stride is None:
            stride = st
        elif st != stride:
            raise ValueError("all x must share one token stride")
        if codes[i].dtype != torch.uint8 or tuple(codes[i].shape) != (L, H, cw) or not codes[i].is_contiguous():
            raise ValueError(f"tensor {i}: codes must be contiguous uint8 {(L, H, cw)}")
        if scales[i].dtype != torch.bfloat16 or tuple(scales[i].shape) != (L, H, n_groups) \
                or not scales[i].is_contiguous():
            raise ValueError(f"tensor {i}: scales must be contiguous bf16 {(L, H, n_groups)}")
        sk = sinks[i] if sinks is not None else None
        if sk is not None and (sk.dtype != torch.bfloat16 or sk.shape[0] < min(sink_tokens, L)
                               or tuple(sk.shape[1:]) != (H, D) or not sk.is_contiguous()):
            raise ValueError(f"tensor {i}: sink must be contiguous bf16 [>=sink_tokens, H, D]")
    cb = _host_map(chan_band)
    if cb.shape[0] != D:
        raise ValueError(f"chan_band has {cb.shape[0]} entries, head_dim is {D}")
    arr = lambda ts: (ctypes.c_void_p * n)(*[_ptr(t) for t in ts])  # noqa: E731
    sink_arr = arr(sinks) if sinks is not None else None
    with torch.cuda.device(dev):
        rc = _lib.load().kvq_rebuild_layers(
            n, ctypes.cast(arr(xs), ctypes.c_void_p), stride, ctypes.cast(arr(codes), ctypes.c_void_p),
            ctypes.cast(arr(scales), ctypes.c_void_p),
            ctypes.cast(sink_arr, ctypes.c_void_p) if sink_arr is not None else None,
            int(sink_tokens) if sinks is not None else 0, L, H, D, cb.ctypes.data_as(ctypes.c_void_p),
            int(n_groups), int(bits), _stream(dev))
    _lib.check(rc, "kvq_rebuild_layers")


def dequantize_into(codes: torch.Tensor, scales: torch.Tensor, out: torch.Tensor, chan_band,
                    n_groups: int, bits: int = 4, sink: torch.Tensor | None = None,
                    sink_tokens: int = 0) -> torch.Tensor:
    """Dequantize codes/scales [L, H, *] into out [L, H, D] bf16 (any token stride)."""
    dev = _require_cuda(codes, scales, out, sink)
    if out.dtype != torch.bfloat16:
        raise TypeError(f"out must be bfloat16, got {out.dtype}")
    L, H, D = out.shape
    os_ = _rows_view_ok(out, "out", D)
    cw = D // 2 if bits == 4 else D
    if codes.dtype != torch.uint8 or tuple(codes.shape) != (L, H, cw) or not codes.is_contiguous():
        raise ValueError(f"codes must be contiguous uint8 {(L, H, cw)}, got {codes.dtype} {tuple(codes.shape)}")
    if scales.dtype != torch.bfloat16 or tuple(scales.shape) != (L, H, n_groups) or not scales.is_contiguous():
        raise ValueError(f"scales must be contiguous bf16 {(L, H, n_groups)}")
    if sink is not None and (sink.dtype != torch.bfloat16 or not sink.is_contiguous()
                             or tuple(sink.shape[1:]) != (H, D) or sink.shape[0] < min(sink_tokens, L)):
        raise ValueError("sink must be contiguous bf16 [>=sink_tokens, H, D]")
    cb = _host_map(chan_band)
    if cb.shape[0] != D:
        raise ValueError(f"chan_band has {cb.shape[0]} entries, head_dim is {D}")
    with torch.cuda.device(dev):
        rc = _lib.load().kvq_dequantize(
            _ptr(codes), _ptr(scales), _ptr(sink), int(sink_tokens) if sink is not None else 0,
            _ptr(out), os_, L, H, D, cb.ctypes.data_as(ctypes.c_void_p), int(n_groups), int(bits),
            _stream(dev))
    _lib.check(rc, "kvq_dequantize")
    return out


def requantize_into(src_codes: torch.Tensor, src_scales: torch.Tensor, dst_codes: torch.Tensor,
                    dst_scales: torch.Tensor, chan_band, n_groups: int, bits: int = 4,
                    exact: torch.Tensor | None = None, exact_tokens: int = 0,
                    sink: torch.Tensor | None = None, sink_tokens: int = 0) -> bool:
    """dst := quantize(dequantize(src)) for packed rows [L, H, *] (kvq_requantize):
    the first exact_tokens source tokens take their bf16 rows from `exact` instead
    of their codes, and the first sink_tokens destination tokens also get the bf16
    rows in `sink`. Returns False, launching nothing, when the fused kernel does not
    cover the format (int8 codes, head_dim other than 128, a generic group map)."""
    dev = _require_cuda(src_codes, src_scales, dst_codes, dst_scales, exact, sink)
    L, H, cw = src_codes.shape
    D = 2 * cw if bits == 4 else cw
    for name, t, shape, dt in (("src_codes", src_codes, (L, H, cw), torch.uint8),
                               ("dst_codes", dst_codes, (L, H, cw), torch.uint8),
                               ("src_scales", src_scales, (L, H, n_groups), torch.bfloat16),
                               ("dst_scales", dst_scales, (L, H, n_groups), torch.bfloat16)):
        if t.dtype != dt or tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous {dt} {shape}, got {t.dtype} {tuple(t.shape)}")
    for name, t, n in (("exact", exact, exact_tokens), ("sink", sink, sink_tokens)):
        if t is not None and (t.dtype != torch.bfloat16 or not t.is_contiguous()
                              or tuple(t.shape[1:]) != (H, D) or t.shape[0] < min(n, L)):
            raise ValueError(f"{name} must be contiguous bf16 [>={name}_tokens, H, D]")
    cb = _host_map(chan_band)
    if cb.shape[0] != D:
        raise ValueError(f"chan_band has {cb.shape[0]} entries, head_dim is {D}")
    with torch.cuda.device(dev):
        rc = _lib.load().kvq_requantize(
            _ptr(src_codes), _ptr(src_scales), _ptr(exact), int(exact_tokens) if exact is not None else 0,
            _ptr(dst_codes), _ptr(dst_scales), _ptr(sink), int(sink_tokens) if sink is not None else 0,
            L, H, D, cb.ctypes.data_as(ctypes.c_void_p), int(n_groups), int(bits), _stream(dev))
    if rc == _lib.KVQ_ERR_UNSUPPORTED:
        return False
    _lib.check(rc, "kvq_requantize")
    return True


# Per (device, stream) workspace of the attention launches (kvq_attention's
# wave-balance parts): grown when a launch needs more, reused in stream order.
_WORKSPACES: dict = {}


def _workspace(dev: torch.device, B: int, Lq: int, H: int, n_kv: int):
    """(pointer, bytes) of a workspace for an attention launch of this shape on the
    current stream of `dev`, or (None, 0) when the launch runs every unit whole."""
    need = ctypes.c_int64()
    with torch.cuda.device(dev):
        _lib.check(_lib.load().kvq_attention_workspace_bytes(B, Lq, H, n_kv, ctypes.byref(need)),
                   "kvq_attention_workspace_bytes")
    if need.value == 0:
        return None, 0
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < need.value:
        buf = torch.empty(need.value + 256, dtype=torch.uint8, device=dev)
        _WORKSPACES[key] = buf
    base = (buf.data_ptr() + 255) // 256 * 256
    return ctypes.c_void_p(base), need.value


def attention_packed(q: torch.Tensor, k_cache, v_cache, lo: int, hi: int, out: torch.Tensor | None = None,
                     softmax_scale: float | None = None, stats: torch.Tensor | None = None) -> torch.Tensor:
    """Fused int4-KV attention of q [B, Lq, H, D] bf16 over tokens [lo, hi) of two
    QuantKVTensor caches (same shape, group mode and sink). Returns out [B, Lq, H, D] bf16.
    With stats (fp32 [B, Lq, H, 4], contiguous) the kernel also writes per row:
    log-sum-exp, entropy (nats), max weight and the mass on the sink tokens."""
    dev = _require_cuda(q, k_cache.packed, v_cache.packed, out)
    if q.dtype != torch.bfloat16 or q.dim() != 4:
        raise TypeError("q must be a [B, Lq, H, D] bfloat16 tensor")
    B, Lq, H, D = q.shape
    for c in (k_cache, v_cache):
        if (c.n_streams, c.n_heads, c.head_dim) != (B, H, D):
            raise ValueError(f"cache shape {tuple(c.shape)} does not match q {tuple(q.shape)}")
    if (k_cache.n_tokens, k_cache.sink_tokens, k_cache.bands) != (v_cache.n_tokens, v_cache.sink_tokens,
                                                                  v_cache.bands):
        raise ValueError("K and V caches must share tokens, sink and group mode")
    if q.stride(3) != 1 or q.stride(2) != D or q.stride(0) != Lq * q.stride(1):
        q = q.contiguous()
    if out is None:
        out = torch.empty((B, Lq, H, D), dtype=torch.bfloat16, device=dev)
    elif (out.dtype != torch.bfloat16 or tuple(out.shape) != (B, Lq, H, D) or out.stride(3) != 1
          or out.stride(2) != D or out.stride(0) != Lq * out.stride(1)):
        raise ValueError("out must be bf16 [B, Lq, H, D] with contiguous heads and a uniform token stride")
    cb = _host_map(k_cache.chan_band_host)
    common = (_ptr(q), q.stride(1), _ptr(k_cache.packed), _ptr(k_cache.scales), _ptr(k_cache.sink),
              _ptr(v_cache.packed), _ptr(v_cache.scales), _ptr(v_cache.sink), k_cache.n_tokens,
              k_cache.sink_tokens if k_cache.sink is not None else 0, int(lo), int(hi), _ptr(out), out.stride(1))
    tail = (B, Lq, H, D, cb.ctypes.data_as(ctypes.c_void_p), len(k_cache.bands), k_cache.bits, v_cache.bits,
            float(softmax_scale) if softmax_scale else 0.0, _stream(dev))
    with torch.cuda.device(dev):
        if stats is None:
            ws, wsb = _workspace(dev, B, Lq, H, int(hi) - int(lo))
            rc = _lib.load().kvq_attention(*common, *tail[:-1], ws, wsb, tail[-1])
        else:
            _require_cuda(stats)
            if stats.dtype != torch.float32 or tuple(stats.shape) != (B, Lq, H, 4) or not stats.is_contiguous():
                raise ValueError(f"stats must be contiguous float32 {(B, Lq, H, 4)}")
            rc = _lib.load().kvq_attention_stats(*common, _ptr(stats), *tail)
    _lib.check(rc, "kvq_attention")
    return out


def attention_timeout_test(q: torch.Tensor, k_cache, v_cache, lo: int, hi: int, stall_tile: int,
                           wait_cycles: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """attention_packed() with the K tiles from `stall_tile` on withheld and every
    bounded wait limited to `wait_cycles` (kvq_test_attention_timeout): the
    launch gives up, raises the device status word and returns; its output is
    invalid. A test hook of the abort path, not a compute entry point."""
    dev = _require_cuda(q, k_cache.packed, v_cache.packed, out)
    B, Lq, H, D = q.shape
    q = q.contiguous()
    if out is None:
        out = torch.empty((B, Lq, H, D), dtype=torch.bfloat16, device=dev)
    cb = _host_map(k_cache.chan_band_host)
    with torch.cuda.device(dev):
        rc = _lib.load().kvq_test_attention_timeout(
            _ptr(q), q.stride(1), _ptr(k_cache.packed), _ptr(k_cache.scales), _ptr(k_cache.sink),
            _ptr(v_cache.packed), _ptr(v_cache.scales), _ptr(v_cache.sink), k_cache.n_tokens,
            k_cache.sink_tokens if k_cache.sink is not None else 0, int(lo), int(hi), _ptr(out), out.stride(1),
            B, Lq, H, D, cb.ctypes.data_as(ctypes.c_void_p), len(k_cache.bands), k_cache.bits, v_cache.bits, 0.0,
            int(stall_tile), int(wait_cycles), _stream(dev))
    _lib.check(rc, "kvq_test_attention_timeout")
    return out


def attention_packed_gather(q: torch.Tensor, k_cache, v_cache, lo: int, hi: int, outs: list[int],
                            out_head0: int, out_heads: int, out_token_stride: int | None = None,
                            softmax_scale: float | None = None) -> None:
    """Head-sharded attention whose epilogue is the output all-gather: the H heads
    of q [B, Lq, H, D] (heads out_head0.. of the full model) are written into each
    of the device buffers `outs` (raw pointers, e.g. PeerOutputs.ptrs: this GPU's
    and its peers'), all laid out [B, Lq, out_heads, D] bf16 with the given token
    stride (default out_heads * D). Every rank's buffer holds the whole output
    once every rank has passed the following gather_barrier()."""
    dev = _require_cuda(q, k_cache.packed, v_cache.packed)
    if q.dtype != torch.bfloat16 or q.dim() != 4:
        raise TypeError("q must be a [B, Lq, H, D] bfloat16 tensor")
    B, Lq, H, D = q.shape
    for c in (k_cache, v_cache):
        if (c.n_streams, c.n_heads, c.head_dim) != (B, H, D):
            raise ValueError(f"cache shape {tuple(c.shape)} does not match q {tuple(q.shape)}")
    if (k_cache.n_tokens, k_cache.sink_tokens, k_cache.bands) != (v_cache.n_tokens, v_cache.sink_tokens,
                                                                  v_cache.bands):
        raise ValueError("K and V caches must share tokens, sink and group mode")
    if not 1 <= len(outs) <= 8:
        raise ValueError(f"1 to 8 output buffers, got {len(outs)}")
    if q.stride(3) != 1 or q.stride(2) != D or q.stride(0) != Lq * q.stride(1):
        q = q.contiguous()
    stride = out_heads * D if out_token_stride is None else int(out_token_stride)
    arr = (ctypes.c_void_p * len(outs))(*[ctypes.c_void_p(int(p)) for p in outs])
    cb = _host_map(k_cache.chan_band_host)
    ws, wsb = _workspace(dev, B, Lq, H, int(hi) - int(lo))
    with torch.cuda.device(dev):
        rc = _lib.load().kvq_attention_gather(
            _ptr(q), q.stride(1), _ptr(k_cache.packed), _ptr(k_cache.scales), _ptr(k_cache.sink),
            _ptr(v_cache.packed), _ptr(v_cache.scales), _ptr(v_cache.sink), k_cache.n_tokens,
            k_cache.sink_tokens if k_cache.sink is not None else 0, int(lo), int(hi),
            ctypes.cast(arr, ctypes.c_void_p), len(outs), int(out_head0), int(out_heads), stride,
            B, Lq, H, D, cb.ctypes.data_as(ctypes.c_void_p), len(k_cache.bands), k_cache.bits, v_cache.bits,
            float(softmax_scale) if softmax_scale else 0.0, ws, wsb, _stream(dev))
    _lib.check(rc, "kvq_attention_gather")


def gather_barrier(counters: list[int], self_index: int, target: int, wait_cycles: int = 2_000_000_000) -> None:
    """Device-side barrier of the ranks on the current stream (kvq_gather_barrier):
    adds 1 to every rank's counter (raw pointers, e.g. PeerOutputs.sig_ptrs) once
    the work before it on the stream has completed, then waits on the device until
    this rank's counter (counters[self_index]) reaches `target` modulo 2^32. Gives
    up after wait_cycles and raises the device status word instead of hanging."""
    n = len(counters)
    arr = (ctypes.c_void_p * n)(*[ctypes.c_void_p(int(p)) for p in counters])
    dev = torch.device("cuda", torch.cuda.current_device())
    rc = _lib.load().kvq_gather_barrier(ctypes.cast(arr, ctypes.c_void_p), n, int(self_index),
                                        ctypes.c_uint(int(target) & 0xFFFFFFFF), int(wait_cycles), _stream(dev))
    _lib.check(rc, "kvq_gather_barrier")


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(handle, byte offset) naming the CUDA allocation that holds t, for
    ipc_import() in another process."""
    _require_cuda(t)
    h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    off = ctypes.c_int64()
    with torch.cuda.device(t.device):
        _lib.check(_lib.load().kvq_ipc_export(_ptr(t), h, ctypes.byref(off)), "kvq_ipc_export")
    return h.raw, off.value


def ipc_import(handle: bytes, offset: int) -> tuple[int, int]:
    """Maps another process's allocation on the current device; returns (base, ptr)."""
    if len(handle) != _lib.IPC_HANDLE_BYTES:
        raise ValueError("bad IPC handle")
    base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
    _lib.check(_lib.load().kvq_ipc_import(handle, int(offset), ctypes.byref(base), ctypes.byref(ptr)),
               "kvq_ipc_import")
    return base.value, ptr.value


def ipc_close(base: int) -> None:
    _lib.check(_lib.load().kvq_ipc_close(ctypes.c_void_p(base)), "kvq_ipc_close")


def device_status(reset: bool = True) -> int:
    """Synchronizes and returns the library's device status word (0 = ok)."""
    rc = _lib.load().kvq_device_status(1 if reset else 0)
    if rc < 0:
        _lib.check(rc, "kvq_device_status")
    return rc
