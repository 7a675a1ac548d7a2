"""Drop-in replacement for the reference's quant_kv_kernels.py on B200 (sm_100a).

Same entry points as sztlink/krea-realtime-bench quant_kv_kernels.py:
  quantize(x, chan_band, G, qmax, dtype)   quant_kv_kernels.py:102-111
  dequantize(packed, scales, chan_band, D, dtype)   quant_kv_kernels.py:91-99
  build_chan_band(bands, D, device)        quant_kv_kernels.py:114-119
  HAVE_TRITON                              quant_kv_kernels.py:23-28
but the kernels are hand-written CUDA for sm_100a behind the libkvq C ABI
(include/kvq.h), not Triton. Differences a caller can see:
  * codes are bit-exact to the reference's torch path (round half to even),
    where the reference's Triton kernel rounds ties away from zero
    (quant_kv_kernels.py:81-82); dequantize is bit-identical to both;
  * there is no CPU path: CPU tensors raise instead of falling back;
  * qmax=127 selects int8 codes ([L, H, D], code = q + 128), the int8 scheme of
    the reference's torch path (quant_kv.py:155-156), which its Triton kernel
    does not cover.
HAVE_TRITON keeps its name because the reference's quant_kv.py gates on it
(quant_kv.py:50-52); here it means "the fused kernels are available" and is
True only when libkvq.so loads.
"""
from __future__ import annotations

import numpy as np
import torch

from kvq import _lib, ops

try:
    _lib.load()
    HAVE_KVQ = True
except Exception:  # the entry points below raise with the load error
    HAVE_KVQ = False
HAVE_TRITON = HAVE_KVQ

# host copies of group maps handed out by build_chan_band, keyed by the device
# tensor's (data_ptr, version); the CUDA kernels specialise on the map's contents,
# which must be known on the host without a device->host sync per launch
_HOST_MAPS: dict = {}


def build_chan_band(bands, D, device):
    """int32 [D] group index per channel on `device` (quant_kv_kernels.py:114-119)."""
    cb = np.zeros(D, dtype=np.int32)
    for gi, (lo, hi) in enumerate(bands):
        cb[lo:hi] = gi
    t = torch.from_numpy(cb.copy()).to(device)
    _HOST_MAPS[(t.data_ptr(), t._version)] = cb
    return t


def host_chan_band(chan_band) -> np.ndarray:
    """Host int32 copy of a group map given as a tensor, array or sequence."""
    if isinstance(chan_band, torch.Tensor):
        if chan_band.device.type == "cpu":
            return np.ascontiguousarray(chan_band.to(torch.int32).numpy())
        key = (chan_band.data_ptr(), chan_band._version)
        hit = _HOST_MAPS.get(key)
        if hit is None:
            hit = np.ascontiguousarray(chan_band.to(torch.int32).cpu().numpy())
            _HOST_MAPS[key] = hit
        return hit
    return np.ascontiguousarray(np.asarray(chan_band, dtype=np.int32))


def _bits_of(qmax) -> int:
    q = int(qmax)
    if q == 7:
        return 4
    if q == 127:
        return 8
    raise ValueError(f"qmax must be 7 (int4) or 127 (int8), got {qmax}")


def quantize(x, chan_band, G, qmax, dtype=torch.bfloat16):
    """x [L,H,D] bf16 -> (packed [L,H,D/2] uint8, scales [L,H,G] bf16).

    Bit-exact to QuantKVTensor._quantize's torch path (quant_kv.py:142-159).
    """
    if dtype != torch.bfloat16:
        raise TypeError(f"only bfloat16 scales are supported, got {dtype}")
    if not isinstance(x, torch.Tensor) or x.dim() != 3:
        raise ValueError("x must be a [L, H, D] tensor")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"x must be bfloat16, got {x.dtype}")
    bits = _bits_of(qmax)
    L, H, D = x.shape
    if x.stride(2) != 1 or x.stride(1) != D or x.data_ptr() % 16 or x.stride(0) % 8:
        x = x.contiguous()
    packed = torch.empty((L, H, D // 2 if bits == 4 else D), dtype=torch.uint8, device=x.device)
    scales = torch.empty((L, H, int(G)), dtype=dtype, device=x.device)
    ops.quantize_into(x, packed, scales, host_chan_band(chan_band), int(G), bits)
    return packed, scales


def dequantize(packed, scales, chan_band, D, dtype=torch.bfloat16):
    """packed [L,H,D/2] uint8 (or [L,H,D] int8 codes), scales [L,H,G] bf16 -> [L,H,D] bf16."""
    if dtype != torch.bfloat16:
        raise TypeError(f"only bfloat16 output is supported, got {dtype}")
    L, H, P = packed.shape
    D = int(D)
    if P == D // 2:
        bits = 4
    elif P == D:
        bits = 8
    else:
        raise ValueError(f"packed last dim {P} matches neither D/2 nor D (D={D})")
    out = torch.empty((L, H, D), dtype=dtype, device=packed.device)
    ops.dequantize_into(packed.contiguous(), scales.contiguous(), out, host_chan_band(chan_band),
                        scales.shape[-1], bits)
    return out
