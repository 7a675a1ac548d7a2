"""Drop-in replacement for the reference's quant_kv.py on B200 (sm_100a).

Same public surface as sztlink/krea-realtime-bench quant_kv.py:
  FRAME_SEQ_LEN, ROPE_BANDS, HAVE_KERNELS, USE_KERNELS   quant_kv.py:50-59
  _band_edges(head_dim, mode)                            quant_kv.py:62-82
  QuantKVTensor(shape, device, dtype, bits, group_mode, sink_tokens)
                                                         quant_kv.py:85-225
  install(pipeline, k_bits, v_bits, group_mode, sink_frames, verbose)
                                                         quant_kv.py:228-269
plus the attention entry point that consumes the cache in packed form,
`attention(q, k, v, ...)`, the call the runtime makes on a cache read
(quant_kv.py:14; hook point probe_attention.py:97-124).

Behaviour a caller can see, against the reference:
  * slice writes quantize on the GPU straight into the cache slice (no
    temporary + copy), codes/scales bit-exact to the reference torch path;
  * slice reads `t[:, a:b]` return a QuantKVWindow, a lazy view of the packed
    window. attention() reads it in packed form; any other use (a torch
    function, a tensor method) dequantizes it exactly as the reference's
    __getitem__ does (quant_kv.py:189-199), sink overlay included;
  * `t[:, a:b].clone()` is a packed snapshot (PackedBlock) with the same bf16
    values as the reference's clone; written into a slice (the eviction
    `kv[:, a:b] = kv[:, c:d].clone()`, quant_kv.py:13) it is requantized in one
    fused pass, bit-exact to the reference's dequantize + quantize;
  * the leading dimension may be > 1: independent streams, each with its own
    window (the reference asserts batch 1, quant_kv.py:95);
  * there is no CPU path (the reference falls back to torch on CPU,
    quant_kv.py:114): a non-CUDA device raises.
"""
from __future__ import annotations

import os
import warnings

import numpy as np
import torch

import quant_kv_kernels as _kern
from kvq import ops as _ops

HAVE_KERNELS = _kern.HAVE_TRITON
# no switch to a non-kernel path exists in this build
USE_KERNELS = HAVE_KERNELS
if os.environ.get("QKV_KERNELS", "1") == "0":
    warnings.warn("QKV_KERNELS=0 is ignored: the B200 build has only the CUDA kernel path")

FRAME_SEQ_LEN = 1560
ROPE_BANDS = ((0, 44), (44, 86), (86, 128))


def _band_edges(head_dim, mode):
    """Channel groups (quant_kv.py:62-82): "bands" = the three rotary bands,
    "bandsN" = each band cut in N pieces on even channels, "blindN" = fixed width."""
    if mode.startswith("bands"):
        assert head_dim == 128, f"rotary bands are mapped for head_dim 128, got {head_dim}"
        n = int(mode[5:]) if len(mode) > 5 else 1
        if n == 1:
            return ROPE_BANDS
        out = []
        for lo, hi in ROPE_BANDS:
            width = hi - lo
            step = max(2, ((width + n - 1) // n + 1) // 2 * 2)
            for s in range(lo, hi, step):
                out.append((s, min(s + step, hi)))
        return tuple(out)
    if mode.startswith("blind"):
        g = int(mode[5:])
        return tuple((i, min(i + g, head_dim)) for i in range(0, head_dim, g))
    raise ValueError(f"unknown group mode: {mode}")


def _token_slice(idx):
    """Accepts [:, a:b] and [:, a:b, ...] (quant_kv.py:179-187)."""
    if not isinstance(idx, tuple):
        raise TypeError("QuantKVTensor expects [:, a:b] indexing")
    assert idx[0] == slice(None), "the batch dimension is always taken whole"
    sl = idx[1]
    assert isinstance(sl, slice) and sl.step in (None, 1), "contiguous slices only"
    return sl


class QuantKVTensor:
    """Behaves like a [B, S, H, D] bf16 tensor across the runtime's operations.

    Storage (reference layout, quant_kv.py:107-111; streams stacked along the
    token axis, stream i owning rows [i*S, (i+1)*S)):
      packed  uint8 [B*S, H, D/2] (int4) or [B*S, H, D] (int8)
      scales  bf16  [B*S, H, G]
      sink    bf16  [B*sink, H, D] or None
    """

    def __init__(self, shape, device, dtype=torch.bfloat16, bits=4,
                 group_mode="bands", sink_tokens=0, lossless_moves=False):
        b, s, h, d = shape
        assert b >= 1, "batch must be >= 1"
        assert bits in (4, 8), "int4 or int8"
        if dtype != torch.bfloat16:
            raise TypeError(f"only bfloat16 caches are supported, got {dtype}")
        dev = torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError(f"QuantKVTensor needs a CUDA (sm_100) device, got {device}; "
                               "the B200 build has no CPU path")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.logical_shape = torch.Size(shape)
        self.dtype = dtype
        self.device = dev
        self.bits = bits
        self.n_streams = b
        self.n_tokens, self.n_heads, self.head_dim = s, h, d
        self.bands = _band_edges(d, group_mode)
        self.group_mode = group_mode
        self.qmax = (1 << (bits - 1)) - 1
        self.sink_tokens = min(sink_tokens, s)
        packed_d = d // 2 if bits == 4 else d
        self.packed = torch.zeros((b * s, h, packed_d), dtype=torch.uint8, device=dev)
        self.scales = torch.zeros((b * s, h, len(self.bands)), dtype=dtype, device=dev)
        self.sink = (torch.zeros((b * self.sink_tokens, h, d), dtype=dtype, device=dev)
                     if self.sink_tokens else None)
        self.use_kernels = True
        # off (the reference's semantics): `kv[:, a:b] = kv[:, c:d].clone()` dequantizes
        # and requantizes the moved tokens (quant_kv.py:217-218, lossy). On: the clone
        # is a snapshot of the packed rows and the write copies codes and scales
        # unchanged (the lossless move README.md:259 describes).
        self.lossless_moves = bool(lossless_moves)
        self.chan_band = _kern.build_chan_band(self.bands, d, dev)
        self.chan_band_host = np.ascontiguousarray(_kern.host_chan_band(self.chan_band))
        # bumped by every write; a window read before a write refuses to be used after it
        self.version = 0

    # ------------------------------------------------------------------ tensor-like
    @property
    def shape(self):
        return self.logical_shape

    def size(self, dim=None):
        return self.logical_shape if dim is None else self.logical_shape[dim]

    def numel(self):
        return int(self.logical_shape.numel())

    def dim(self):
        return 4

    def zero_(self):
        self.version += 1
        self.packed.zero_()
        self.scales.zero_()
        if self.sink is not None:
            self.sink.zero_()
        return self

    def storage_bytes(self):
        n = self.packed.numel() + self.scales.numel() * self.scales.element_size()
        if self.sink is not None:
            n += self.sink.numel() * self.sink.element_size()
        return n

    # ------------------------------------------------------------------ quant / dequant
    def _quantize(self, x):
        """x [L, H, D] bf16 -> (packed, scales), new tensors (quant_kv.py:142-159)."""
        return _kern.quantize(x, self.chan_band, len(self.bands), self.qmax, self.dtype)

    def _dequantize(self, packed, scales):
        """(packed, scales) -> [L, H, D] bf16 (quant_kv.py:161-176)."""
        return _kern.dequantize(packed, scales, self.chan_band, self.head_dim, self.dtype)

    # ------------------------------------------------------------------ stream rows
    def _rows(self, stream, a, b):
        o = stream * self.n_tokens
        return slice(o + a, o + b)

    def _sink_rows(self, stream, a, b):
        o = stream * self.sink_tokens
        return slice(o + a, o + b)

    def write_(self, a, b, value):
        """Quantize value [B, b-a, H, D] (or [b-a, H, D] when B == 1) into tokens [a, b)."""
        v = value
        if v.dim() == 3:
            v = v.unsqueeze(0)
        assert v.dim() == 4 and v.shape[0] == self.n_streams, \
            f"value has {v.shape[0]} streams, cache has {self.n_streams}"
        assert v.shape[1] == b - a, f"write of {v.shape[1]} tokens into a slice of {b - a}"
        if v.dtype != self.dtype:
            v = v.to(self.dtype)
        if v.device != self.device:
            v = v.to(self.device)
        _write_tensors([(self, v)], a, b)

    def write_rope_(self, a, b, value, freqs, positions):
        """Slice write [a, b) of keys before their rotary embedding, rotated in the
        quantize kernel (kvq_rope_quantize): value [B, b-a, H, 128] bf16, freqs
        [P, 64, 2] float64 on the cache's device (kvq.rope.freqs), positions
        [b-a, 3] int32 (frame, height, width; kvq.rope.grid_positions), shared by
        the streams. Equal to writing the rotated keys (quant_kv.py:201-215)."""
        v = value.unsqueeze(0) if value.dim() == 3 else value
        assert v.dim() == 4 and v.shape[0] == self.n_streams and v.shape[1] == b - a
        v = v.to(device=self.device, dtype=self.dtype)
        self.version += 1
        freqs = freqs.to(self.device).contiguous()
        positions = positions.to(device=self.device, dtype=torch.int32).contiguous()
        G = len(self.bands)
        ns = max(0, min(b, self.sink_tokens) - a) if self.sink is not None else 0
        for i in range(self.n_streams):
            x = v[i]
            if x.stride(2) != 1 or x.stride(1) != self.head_dim or x.data_ptr() % 16 or x.stride(0) % 8:
                x = x.contiguous()
            rows = self._rows(i, a, b)
            sink = self.sink[self._sink_rows(i, a, a + ns)] if ns > 0 else None
            _ops.rope_quantize_into(x, self.packed[rows], self.scales[rows], self.chan_band_host, G, self.bits,
                                    freqs, positions, sink=sink, sink_tokens=ns)

    def read(self, a, b, out=None):
        """Dequantize tokens [a, b) with the sink overlay -> [B, b-a, H, D] bf16."""
        B, H, D = self.n_streams, self.n_heads, self.head_dim
        if out is None:
            out = torch.empty((B, b - a, H, D), dtype=self.dtype, device=self.device)
        ns = max(0, min(b, self.sink_tokens) - a) if self.sink is not None else 0
        for i in range(B):
            rows = self._rows(i, a, b)
            sink = self.sink[self._sink_rows(i, a, a + ns)] if ns > 0 else None
            _ops.dequantize_into(self.packed[rows], self.scales[rows], out[i], self.chan_band_host,
                                 len(self.bands), self.bits, sink=sink, sink_tokens=ns)
        return out

    # ------------------------------------------------------------------ slicing
    def __getitem__(self, idx):
        sl = _token_slice(idx)
        a, b, _ = sl.indices(self.n_tokens)
        if b <= a:
            return torch.empty((self.n_streams, 0, self.n_heads, self.head_dim),
                               dtype=self.dtype, device=self.device)
        return QuantKVWindow(self, a, b)

    def __setitem__(self, idx, value):
        sl = _token_slice(idx)
        a, b, _ = sl.indices(self.n_tokens)
        if b <= a:
            return
        if isinstance(value, PackedBlock) and value.fits(self, b - a):
            if self.lossless_moves:
                self.write_packed_(a, b, value)
                return
            if self.write_requant_(a, b, value):
                return
        if isinstance(value, QuantKVWindow):
            value = value.materialize()
        self.write_(a, b, value)

    def write_packed_(self, a, b, blk):
        """Tokens [a, b) := the packed rows of blk (codes and scales copied as they
        are); destination tokens below sink_tokens also get blk's bf16 read values
        in the sink (exact where blk's rows came from its cache's sink)."""
        L = b - a
        ns = max(0, min(b, self.sink_tokens) - a) if self.sink is not None else 0
        self.version += 1
        for i in range(self.n_streams):
            rows = self._rows(i, a, b)
            self.packed[rows].copy_(blk.packed[i * L:(i + 1) * L])
            self.scales[rows].copy_(blk.scales[i * L:(i + 1) * L])
            if ns > 0:
                self.sink[self._sink_rows(i, a, a + ns)].copy_(blk.read_rows(i, 0, ns))

    def write_requant_(self, a, b, blk) -> bool:
        """Tokens [a, b) := quantize(blk's bf16 read), as the reference's slice write of
        a cloned window does (quant_kv.py:13, 201-215), in one fused pass over blk's
        packed rows (kvq_requantize): no bf16 window is materialized. Destination
        tokens below sink_tokens also get the bf16 values in the sink. Returns False,
        writing nothing, for a format the fused kernel does not cover."""
        L = b - a
        if self.bits != 4 or self.head_dim != 128:
            return False
        ns = max(0, min(b, self.sink_tokens) - a) if self.sink is not None else 0
        for i in range(self.n_streams):
            rows = self._rows(i, a, b)
            exact = blk.exact[i] if blk.n_exact > 0 else None
            sink = self.sink[self._sink_rows(i, a, a + ns)] if ns > 0 else None
            done = _ops.requantize_into(blk.packed[i * L:(i + 1) * L], blk.scales[i * L:(i + 1) * L],
                                        self.packed[rows], self.scales[rows], self.chan_band_host,
                                        len(self.bands), self.bits, exact=exact, exact_tokens=blk.n_exact,
                                        sink=sink, sink_tokens=ns)
            if not done:
                assert i == 0, "the fused requantize covers every stream of a cache or none"
                return False
            self.version += 1
        return True

    def clone(self):
        raise RuntimeError("QuantKVTensor.clone(): the runtime only clones windows (t[:, a:b].clone()); "
                           "copying a whole packed cache is not supported")

    def __repr__(self):
        return (f"<QuantKVTensor {list(self.logical_shape)} int{self.bits} groups={self.group_mode} "
                f"({len(self.bands)}) sink_tokens={self.sink_tokens} on {self.device}: "
                f"{self.storage_bytes() / 2**30:.2f} GiB resident>")


def attention_stats(q, k, v, softmax_scale=None):
    """attention() plus per-row statistics of the attention distribution, from the
    same fused kernel: returns (out [B, Lq, H, D] bf16, stats [B, Lq, H, 4] fp32)
    with stats[..., 0] = log-sum-exp of the scaled logits, [..., 1] = entropy
    -sum p ln p (nats), [..., 2] = max p, [..., 3] = attention mass on the sink
    tokens. The reference's probe computes entropia / peso_max / massa_ancora the
    same way on a sample of queries (probe_attention.py:102-121)."""
    if not isinstance(k, QuantKVWindow) or not isinstance(v, QuantKVWindow) \
            or isinstance(k, PackedBlock) or isinstance(v, PackedBlock):
        raise TypeError("attention_stats() takes k and v as QuantKVTensor windows (t[:, lo:hi])")
    if (k.lo, k.hi) != (v.lo, v.hi):
        raise ValueError(f"k window [{k.lo},{k.hi}) and v window [{v.lo},{v.hi}) differ")
    k.check_fresh()
    v.check_fresh()
    B, Lq, H, _ = q.shape
    stats = torch.empty((B, Lq, H, 4), dtype=torch.float32, device=k.cache.device)
    out = _ops.attention_packed(q, k.cache, v.cache, k.lo, k.hi, softmax_scale=softmax_scale, stats=stats)
    return out, stats


def _write_tensors(pairs, a, b):
    """Quantize each value [B, b-a, H, D] into tokens [a, b) of its cache, all
    (cache, stream) tensors of one shape in as few launches as possible (96
    tensors per kvq_rebuild_layers launch)."""
    c0 = pairs[0][0]
    G = len(c0.bands)
    ns = max(0, min(b, c0.sink_tokens) - a) if c0.sink is not None else 0
    xs, codes, scales, sinks = [], [], [], []
    for cache, v in pairs:
        cache.version += 1
        for i in range(cache.n_streams):
            x = v[i]
            if x.stride(2) != 1 or x.stride(1) != cache.head_dim or x.data_ptr() % 16 or x.stride(0) % 8:
                x = x.contiguous()
            rows = cache._rows(i, a, b)
            xs.append(x)
            codes.append(cache.packed[rows])
            scales.append(cache.scales[rows])
            sinks.append(cache.sink[cache._sink_rows(i, a, a + ns)] if ns > 0 else None)
    # one token stride per launch: group the tensors by stride
    by_stride = {}
    for k, x in enumerate(xs):
        by_stride.setdefault(x.stride(0), []).append(k)
    for idx in by_stride.values():
        for s0 in range(0, len(idx), 96):
            part = idx[s0:s0 + 96]
            _ops.quantize_layers_into([xs[k] for k in part], [codes[k] for k in part], [scales[k] for k in part],
                                      c0.chan_band_host, G, c0.bits,
                                      sinks=[sinks[k] for k in part] if ns > 0 else None, sink_tokens=ns)


def write_layers(caches, values, a: int, b: int) -> None:
    """caches[i][:, a:b] = values[i] for several caches of one shape, group mode,
    bits and sink (the 40 layers x {K, V} of a rebuild or an append), with one
    launch per 96 (cache, stream) tensors instead of one per tensor. Bit-identical
    to the slice writes (quant_kv.py:201-215 in a loop)."""
    caches, values = list(caches), list(values)
    if len(caches) != len(values) or not caches:
        raise ValueError("one value per cache")
    c0 = caches[0]
    key = lambda c: (tuple(c.logical_shape), c.bits, tuple(c.bands), c.sink_tokens, c.sink is None,  # noqa: E731
                     c.dtype, c.device)
    if any(key(c) != key(c0) for c in caches):
        raise ValueError("write_layers needs caches of one shape, group mode, bits and sink")
    a, b, _ = slice(a, b).indices(c0.n_tokens)
    if b <= a:
        return
    pairs = []
    for c, v in zip(caches, values):
        if isinstance(v, QuantKVWindow):
            v = v.materialize()
        if v.dim() == 3:
            v = v.unsqueeze(0)
        assert v.dim() == 4 and v.shape[0] == c.n_streams and v.shape[1] == b - a, \
            f"value of shape {tuple(v.shape)} for a write of tokens [{a}, {b}) of {c.n_streams} streams"
        if v.dtype != c.dtype:
            v = v.to(c.dtype)
        if v.device != c.device:
            v = v.to(c.device)
        pairs.append((c, v))
    _write_tensors(pairs, a, b)


def _materialize_args(x):
    if isinstance(x, QuantKVWindow):
        return x.materialize()
    if isinstance(x, (list, tuple)):
        return type(x)(_materialize_args(y) for y in x)
    if isinstance(x, dict):
        return {k: _materialize_args(v) for k, v in x.items()}
    return x


class QuantKVWindow:
    """Lazy [B, hi-lo, H, D] bf16 view of tokens [lo, hi) of a QuantKVTensor.

    attention() consumes it packed. Everything else sees the dequantized bf16
    window of the reference's __getitem__ (quant_kv.py:189-199), materialized on
    use: torch functions (via __torch_function__), tensor methods and
    attributes (delegated) and arithmetic operators; `.clone()` takes a packed
    snapshot (PackedBlock) of the same values.

    One difference to the reference, whose __getitem__ returns a snapshot: the
    window is read when it is used, not when it is taken. So that this can never
    return newer data silently, a window refuses to be used (RuntimeError) once
    its cache has been written after the window was taken; take the window
    again, or `.clone()` it before the write to keep the old contents (the clone
    is a packed snapshot, PackedBlock). The runtime's three patterns
    (quant_kv.py:12-14) always use a window at once.
    """

    def __init__(self, cache: QuantKVTensor, lo: int, hi: int):
        self.cache, self.lo, self.hi = cache, lo, hi
        self.version = cache.version

    def check_fresh(self):
        if self.cache.version != self.version:
            raise RuntimeError(f"window [{self.lo}, {self.hi}) of {self.cache!r} was taken before a later write "
                               "to the cache; take it again (or clone() it before writing)")

    @property
    def shape(self):
        c = self.cache
        return torch.Size((c.n_streams, self.hi - self.lo, c.n_heads, c.head_dim))

    @property
    def dtype(self):
        return self.cache.dtype

    @property
    def device(self):
        return self.cache.device

    def size(self, dim=None):
        return self.shape if dim is None else self.shape[dim]

    def dim(self):
        return 4

    def materialize(self) -> torch.Tensor:
        self.check_fresh()
        return self.cache.read(self.lo, self.hi)

    def clone(self, *a, **kw):
        # the runtime's eviction `kv[:, a:b] = kv[:, c:d].clone()` (quant_kv.py:13): the
        # reference dequantizes here and requantizes on the write (quant_kv.py:217-218).
        # The clone is a packed snapshot of the window; written into a cache slice it
        # is requantized in one fused pass (or, with lossless_moves, copied as it is),
        # and any other use sees the same bf16 values as the reference's clone.
        self.check_fresh()
        return PackedBlock(self.cache, self.lo, self.hi)

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        return func(*_materialize_args(args), **_materialize_args(kwargs or {}))

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return getattr(self.materialize(), name)

    def __getitem__(self, idx):
        return self.materialize()[idx]

    def __len__(self):
        return self.cache.n_streams

    def __array__(self, dtype=None):
        return np.asarray(self.materialize().float().cpu(), dtype=dtype)

    def __repr__(self):
        return f"QuantKVWindow({self.cache!r}, tokens [{self.lo}, {self.hi}))"


class PackedBlock(QuantKVWindow):
    """Snapshot of tokens [lo, hi) of a QuantKVTensor in packed form (codes,
    scales, and the bf16 sink rows the window overlaps), made by clone() of a
    window. Writing it into a slice of a cache of the same format requantizes its
    bf16 read in one fused pass, as the reference's write of the dequantized clone
    does (with lossless_moves: copies the packed rows unchanged); any other use sees
    the window's bf16 read (dequantize + sink overlay) as of the snapshot, which is
    what the reference's clone holds. Unlike that clone it is not a torch.Tensor."""

    def __init__(self, cache: QuantKVTensor, lo: int, hi: int):
        super().__init__(cache, lo, hi)
        L = hi - lo
        # torch.cat allocates its result, so the snapshot is one copy of the rows
        self.packed = torch.cat([cache.packed[cache._rows(i, lo, hi)] for i in range(cache.n_streams)]) \
            if L > 0 else cache.packed[:0].clone()
        self.scales = torch.cat([cache.scales[cache._rows(i, lo, hi)] for i in range(cache.n_streams)]) \
            if L > 0 else cache.scales[:0].clone()
        self.n_exact = max(0, min(hi, cache.sink_tokens) - lo) if cache.sink is not None else 0
        self.exact = (torch.stack([cache.sink[cache._sink_rows(i, lo, lo + self.n_exact)]
                                   for i in range(cache.n_streams)]).clone() if self.n_exact > 0 else None)

    def fits(self, cache: QuantKVTensor, n: int) -> bool:
        c = self.cache
        return (n == self.hi - self.lo and cache.bits == c.bits and tuple(cache.bands) == tuple(c.bands)
                and (cache.n_streams, cache.n_heads, cache.head_dim) == (c.n_streams, c.n_heads, c.head_dim)
                and cache.device == c.device)

    def read_rows(self, stream: int, a: int, b: int) -> torch.Tensor:
        """bf16 read of block tokens [a, b) of one stream -> [b-a, H, D]."""
        c, L = self.cache, self.hi - self.lo
        out = torch.empty((b - a, c.n_heads, c.head_dim), dtype=c.dtype, device=c.device)
        if b <= a:
            return out
        rows = slice(stream * L + a, stream * L + b)
        _ops.dequantize_into(self.packed[rows], self.scales[rows], out, c.chan_band_host, len(c.bands), c.bits)
        e = min(b, self.n_exact)
        if e > a:
            out[: e - a].copy_(self.exact[stream, a:e])
        return out

    def materialize(self) -> torch.Tensor:
        L = self.hi - self.lo
        return torch.stack([self.read_rows(i, 0, L) for i in range(self.cache.n_streams)])

    def clone(self, *a, **kw):
        return self

    def __repr__(self):
        return f"PackedBlock({self.cache!r}, tokens [{self.lo}, {self.hi}))"


def _binop(name):
    def f(self, other):
        return getattr(self.materialize(), name)(_materialize_args(other))
    f.__name__ = name
    return f


for _n in ("__add__", "__radd__", "__sub__", "__rsub__", "__mul__", "__rmul__", "__truediv__",
           "__rtruediv__", "__matmul__", "__rmatmul__", "__eq__", "__ne__", "__lt__", "__le__",
           "__gt__", "__ge__"):
    setattr(QuantKVWindow, _n, _binop(_n))
for _n in ("__neg__", "__abs__", "__float__"):
    setattr(QuantKVWindow, _n, (lambda nm: lambda self: getattr(self.materialize(), nm)())(_n))
QuantKVWindow.__hash__ = object.__hash__


def install(pipeline, k_bits=4, v_bits=4, group_mode="bands", sink_frames=0, verbose=True,
            lossless_moves=False):
    """Swaps the kv_cache1 allocation for QuantKVTensor (quant_kv.py:228-269).

    Patches the instance's `_initialize_kv_cache`; the cross-attention cache is
    not touched. Returns the original method. lossless_moves (off by default,
    as in the reference) makes the runtime's eviction copy packed rows instead
    of requantizing them.
    """
    sink_tokens = sink_frames * FRAME_SEQ_LEN
    orig = pipeline._initialize_kv_cache

    def _initialize_kv_cache(batch_size, dtype, device):
        if pipeline.local_attn_size != -1:
            size = pipeline.local_attn_size * pipeline.frame_seq_length
        else:
            size = 32760
        cfg = pipeline.generator.model.config
        shape = [batch_size, size, cfg.num_heads, cfg.dim // cfg.num_heads]
        existing = getattr(pipeline, "kv_cache1", None)
        if existing and isinstance(existing[0]["k"], QuantKVTensor) \
                and list(existing[0]["k"].shape) == shape:
            for e in existing:
                e["k"].zero_()
                e["v"].zero_()
                e["global_end_index"] = 0
                e["local_end_index"] = 0
            return
        cache = []
        extra = {"lossless_moves": True} if lossless_moves else {}  # the reference's call when off
        for _ in range(pipeline.num_transformer_blocks):
            cache.append({
                "k": QuantKVTensor(shape, device, dtype, k_bits, group_mode, sink_tokens, **extra),
                "v": QuantKVTensor(shape, device, dtype, v_bits, group_mode, sink_tokens, **extra),
                "global_end_index": 0,
                "local_end_index": 0,
            })
        pipeline.k_shape = shape
        pipeline.v_shape = shape
        pipeline.kv_cache1 = cache
        if verbose:
            packed = sum(e["k"].storage_bytes() + e["v"].storage_bytes() for e in cache)
            dense = 2 * len(cache) * shape[0] * shape[1] * shape[2] * shape[3] * 2
            print(f"[quant_kv] {len(cache)} layers x (K int{k_bits}, V int{v_bits}), window {shape[1]} tokens, "
                  f"groups {group_mode}, sink {sink_tokens}: {packed / 2**30:.2f} GiB packed, "
                  f"{dense / 2**30:.2f} GiB as bf16", flush=True)

    pipeline._initialize_kv_cache = _initialize_kv_cache
    return orig


# The upstream attention wrapper's optional arguments after (q, k, v), in its
# positional order (Wan's flash-attention wrapper; un-vendored, the reference's
# probe forwards them unchanged, probe_attention.py:101,122).
_UPSTREAM_ARGS = ("q_lens", "k_lens", "dropout_p", "softmax_scale", "q_scale", "causal", "window_size",
                  "deterministic", "dtype", "fa_version")


def _check_lens(lens, n, name):
    if lens is None:
        return
    vals = lens.tolist() if isinstance(lens, torch.Tensor) else list(lens)
    if any(int(x) != n for x in vals):
        raise NotImplementedError(f"{name} other than the full length {n} (variable-length batches) "
                                  "is not supported by the fused int4-KV attention")


def attention(q, k, v, *args, out=None, **kwargs):
    """Attention over a cache read, consuming the packed window directly.

    The runtime's read path `attention(q, kv_cache["k"][:, lo:hi],
    kv_cache["v"][:, lo:hi])` (quant_kv.py:14) with q [B, Lq, H, D] bf16 and k, v
    QuantKVWindow views of the same token range. Non-causal softmax(q k^T *
    scale) v, scale 1/sqrt(D) by default, bf16 output [B, Lq, H, D]. Plain
    tensors for k or v raise TypeError: this build has no non-packed path.

    The upstream wrapper's optional arguments are accepted, positionally or by
    name, when they leave this computation unchanged: q_lens / k_lens equal to
    the full lengths (or None), dropout_p 0, softmax_scale (used), q_scale None,
    causal False, window_size (-1, -1), deterministic (the kernel is), dtype
    bf16, fa_version (ignored). Anything else raises NotImplementedError rather
    than computing something different; unknown names raise TypeError.
    """
    if not isinstance(k, QuantKVWindow) or not isinstance(v, QuantKVWindow) \
            or isinstance(k, PackedBlock) or isinstance(v, PackedBlock):
        raise TypeError("attention() takes k and v as QuantKVTensor windows (t[:, lo:hi]); "
                        "plain tensors and clones have no packed form in the cache")
    if (k.lo, k.hi) != (v.lo, v.hi):
        raise ValueError(f"k window [{k.lo},{k.hi}) and v window [{v.lo},{v.hi}) differ")
    if len(args) > len(_UPSTREAM_ARGS):
        raise TypeError(f"attention() takes at most {3 + len(_UPSTREAM_ARGS)} positional arguments")
    opts = dict(zip(_UPSTREAM_ARGS, args))
    for name, val in kwargs.items():
        if name not in _UPSTREAM_ARGS:
            raise TypeError(f"attention() got an unexpected keyword argument {name!r}")
        if name in opts:
            raise TypeError(f"attention() got multiple values for argument {name!r}")
        opts[name] = val
    k.check_fresh()
    v.check_fresh()
    _check_lens(opts.get("q_lens"), q.shape[1], "q_lens")
    _check_lens(opts.get("k_lens"), k.hi - k.lo, "k_lens")
    if float(opts.get("dropout_p") or 0.0) != 0.0:
        raise NotImplementedError("dropout is not supported by the fused int4-KV attention")
    if opts.get("q_scale") is not None:
        raise NotImplementedError("q_scale is not supported by the fused int4-KV attention")
    if opts.get("causal", False):
        raise NotImplementedError("the cache read is non-causal; causal=True is not supported")
    ws = opts.get("window_size", (-1, -1))
    if ws is not None and tuple(int(x) for x in ws) != (-1, -1):
        raise NotImplementedError("local window_size is not supported by the fused int4-KV attention")
    dt = opts.get("dtype", torch.bfloat16)
    if dt is not None and dt != torch.bfloat16:
        raise NotImplementedError(f"output dtype {dt} is not supported (bf16 only)")
    return _ops.attention_packed(q, k.cache, v.cache, k.lo, k.hi, out=out, softmax_scale=opts.get("softmax_scale"))
