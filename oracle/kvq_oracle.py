"""CPU oracle for the 4-bit KV-cache hot path (test infrastructure only).

This module is the checker, not the product. Only the tests, the smoke check
and the CPU-baseline leg of the benchmark may import it; the CUDA library
never routes through it.

It restates, in numpy on bf16 bit patterns, the reference torch path of
sztlink/krea-realtime-bench:

  band_edges        quant_kv.py:62-82           rotary-band channel groups
  chan_band         quant_kv_kernels.py:114-119 per-channel group index
  quantize          quant_kv.py:142-159         symmetric absmax int4/int8 codes
  dequantize        quant_kv.py:161-176         codes x bf16 scale -> bf16
  QuantKVRef        quant_kv.py:85-225          sink-aware slice write / read
  attention_fp32    upstream attention() as hooked at probe_attention.py:102-124,
                    restated as softmax(q k^T / sqrt(D)) v in fp32

Arithmetic contract (what bit-exactness means here):
  * amax is taken over fp32 copies of bf16 values, scale = amax / qmax as an
    IEEE fp32 divide, scale = 1 where amax == 0 (quant_kv.py:151-152);
  * codes use the UNROUNDED fp32 scale: round-half-to-even(x / s) with an
    IEEE fp32 divide, clamped to [-qmax, qmax] (quant_kv.py:153);
  * the stored scale is bf16(s) with round-to-nearest-even (quant_kv.py:154);
  * int4 codes are offset by +8 and packed two per byte, channel 2i in the
    low nibble and 2i+1 in the high nibble (quant_kv.py:158-159);
  * dequant is bf16(float(code - 8) * float(bf16 scale)) (quant_kv.py:170-175).
Non-finite inputs (NaN/Inf) are outside the contract: the reference's own
result for them depends on the platform's float->int16 conversion.

The oracle is pinned by tests/golden/*.npz, which were produced by importing
the reference itself (tests/golden/make_golden.py).
"""
from __future__ import annotations

import math

import numpy as np

FRAME_SEQ_LEN = 1560                                  # quant_kv.py:57
ROPE_BANDS = ((0, 44), (44, 86), (86, 128))          # quant_kv.py:59


# ----------------------------------------------------------------------------- bf16 bits
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact widening)."""
    b = np.asarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bits, round-to-nearest-even; NaN -> 0x7FC0.

    Same rounding as torch's float -> bfloat16 cast (c10 round_to_nearest_even).
    """
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    bias = np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))
    out = ((u + bias) >> np.uint64(16)).astype(np.uint16)
    return np.where(np.isnan(f), np.uint16(0x7FC0), out).astype(np.uint16)


# ----------------------------------------------------------------------------- groups
def band_edges(head_dim: int, mode: str) -> tuple:
    """Channel groups of a mode (restates quant_kv.py:62-82).

    "bands"  = the three rotary bands [0,44) [44,86) [86,128);
    "bandsN" = each band cut into pieces of an even step that never cross a band;
    "blindN" = fixed groups of N channels.
    """
    if mode.startswith("bands"):
        if head_dim != 128:
            raise AssertionError(f"rotary bands are mapped for head_dim 128, got {head_dim}")
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


def chan_band(bands, head_dim: int) -> np.ndarray:
    """int32 [D] group index per channel (restates quant_kv_kernels.py:114-119)."""
    cb = np.zeros(head_dim, dtype=np.int32)
    for gi, (lo, hi) in enumerate(bands):
        cb[lo:hi] = gi
    return cb


# ----------------------------------------------------------------------------- quant / dequant
def quantize(x_bits: np.ndarray, bands, bits: int = 4):
    """[L, H, D] bf16 bits -> (codes uint8, scales bf16 bits [L, H, G]).

    Restates QuantKVTensor._quantize, torch path (quant_kv.py:142-159).
    int4: codes are [L, H, D/2] packed nibbles; int8: [L, H, D] offset by 128.
    """
    x = bf16_to_f32(x_bits)
    L, H, D = x.shape
    qmax = (1 << (bits - 1)) - 1
    q = np.empty((L, H, D), dtype=np.int16)
    scales = np.empty((L, H, len(bands)), dtype=np.uint16)
    with np.errstate(invalid="ignore"):
        for bi, (lo, hi) in enumerate(bands):
            seg = x[..., lo:hi]
            s = np.abs(seg).max(axis=-1, keepdims=True) / np.float32(qmax)
            s = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
            q[..., lo:hi] = np.clip(np.round(seg / s), -qmax, qmax).astype(np.int16)
            scales[..., bi] = f32_to_bf16(s[..., 0])
    if bits == 8:
        return np.clip(q + 128, 0, 255).astype(np.uint8), scales
    u = np.clip(q + 8, 0, 15).astype(np.uint8)
    return np.ascontiguousarray(u[..., 0::2] | (u[..., 1::2] << np.uint8(4))), scales


def dequantize(codes: np.ndarray, scales_bits: np.ndarray, bands, head_dim: int,
               bits: int = 4) -> np.ndarray:
    """(codes, bf16 scales) -> [L, H, D] bf16 bits (restates quant_kv.py:161-176)."""
    if bits == 8:
        q = codes.astype(np.int16) - 128
    else:
        L, H, P = codes.shape
        q = np.empty((L, H, P * 2), dtype=np.int16)
        q[..., 0::2] = (codes & 0x0F).astype(np.int16) - 8
        q[..., 1::2] = ((codes >> 4) & 0x0F).astype(np.int16) - 8
    sc = bf16_to_f32(scales_bits)
    out = np.empty(q.shape, dtype=np.uint16)
    for bi, (lo, hi) in enumerate(bands):
        out[..., lo:hi] = f32_to_bf16(q[..., lo:hi].astype(np.float32) * sc[..., bi:bi + 1])
    return out


# ----------------------------------------------------------------------------- proxy tensor
class QuantKVRef:
    """Storage semantics of QuantKVTensor (quant_kv.py:85-225) on numpy arrays.

    Shape [1, S, H, D]; storage codes [S, H, D/2 or D], scales [S, H, G] and
    an optional bf16 copy of the first `sink_tokens` rows.
    """

    def __init__(self, S: int, H: int, D: int, bits: int = 4, group_mode: str = "bands",
                 sink_tokens: int = 0):
        self.S, self.H, self.D, self.bits = S, H, D, bits
        self.bands = band_edges(D, group_mode)
        self.sink_tokens = min(sink_tokens, S)
        pd = D // 2 if bits == 4 else D
        self.packed = np.zeros((S, H, pd), np.uint8)
        self.scales = np.zeros((S, H, len(self.bands)), np.uint16)
        self.sink = np.zeros((self.sink_tokens, H, D), np.uint16) if self.sink_tokens else None

    def zero_(self):
        """quant_kv.py:129-133."""
        self.packed[:] = 0
        self.scales[:] = 0
        if self.sink is not None:
            self.sink[:] = 0
        return self

    def setitem(self, a: int, b: int, value_bits: np.ndarray):
        """Slice write [:, a:b] = value (quant_kv.py:201-215)."""
        a, b, _ = slice(a, b).indices(self.S)
        if b <= a:
            return
        v = value_bits[0] if value_bits.ndim == 4 else value_bits
        assert v.shape[0] == b - a
        self.packed[a:b], self.scales[a:b] = quantize(v, self.bands, self.bits)
        if self.sink is not None and a < self.sink_tokens:
            end = min(b, self.sink_tokens)
            self.sink[a:end] = v[: end - a]

    def getitem(self, a: int, b: int) -> np.ndarray:
        """Slice read [:, a:b] -> [1, b-a, H, D] bf16 bits (quant_kv.py:189-199)."""
        a, b, _ = slice(a, b).indices(self.S)
        if b <= a:
            return np.empty((1, 0, self.H, self.D), np.uint16)
        out = dequantize(self.packed[a:b], self.scales[a:b], self.bands, self.D, self.bits)
        if self.sink is not None and a < self.sink_tokens:
            end = min(b, self.sink_tokens)
            out[: end - a] = self.sink[a:end]
        return out[None]


# ----------------------------------------------------------------------------- attention
def attention_fp32(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray,
                   scale: float | None = None) -> np.ndarray:
    """softmax(q k^T * scale) v in fp32, per head, non-causal.

    q [B, Lq, H, D], k/v [B, Lk, H, D] as bf16 bits -> fp32 [B, Lq, H, D].
    The upstream attention() that consumes the dequantized window is an
    un-vendored library call; its math is restated from
    probe_attention.py:111-112 (logits = q k^T / sqrt(D), softmax over keys).
    """
    q = bf16_to_f32(q_bits).astype(np.float32)
    k = bf16_to_f32(k_bits).astype(np.float32)
    v = bf16_to_f32(v_bits).astype(np.float32)
    B, Lq, H, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = np.empty((B, Lq, H, D), np.float32)
    for b in range(B):
        for h in range(H):
            s = (q[b, :, h, :] @ k[b, :, h, :].T) * np.float32(scale)
            s = s - s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=-1, keepdims=True)
            out[b, :, h, :] = p @ v[b, :, h, :]
    return out


# ----------------------------------------------------------------------------- rotary embedding
ROPE_SPLIT = (22, 21, 21)  # complex pairs per axis (frame, height, width) for head_dim 128


def rope_f64(x_bits: np.ndarray, freqs: np.ndarray, pos: np.ndarray) -> np.ndarray:
    """Rotary embedding of bf16 keys [L, H, 128] as the upstream runtime applies it
    before the cache write (Wan's rope_apply; not vendored in the reference, whose
    band split is cited at quant_kv.py:26-31 and bench_qkv.py:64-65): pairs
    (2i, 2i+1) as complex128 numbers times freqs[pos[t][axis(i)], i] = (cos, sin),
    the product's real and imaginary parts rounded to float32 (the upstream
    result) and then to bf16 (the cache dtype). freqs: [P, 64, 2] float64;
    pos: [L, 3] int (frame, height, width); axis(i) = 0, 1, 2 for pairs
    [0, 22), [22, 43), [43, 64). Separate IEEE fp64 products and sums."""
    x = bf16_to_f32(x_bits).astype(np.float64)
    L, H, D = x.shape
    assert D == 128
    x0, x1 = x[..., 0::2], x[..., 1::2]                      # [L, H, 64]
    axis = np.repeat(np.arange(3), ROPE_SPLIT)               # [64]
    p = np.clip(np.asarray(pos, dtype=np.int64), 0, freqs.shape[0] - 1)[:, axis]   # [L, 64]
    cs = freqs[p, np.arange(64)[None, :]]                    # [L, 64, 2]
    c, s = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
    y0 = x0 * c - x1 * s
    y1 = x0 * s + x1 * c
    y = np.empty_like(x)
    y[..., 0::2], y[..., 1::2] = y0, y1
    return f32_to_bf16(y.astype(np.float32))
