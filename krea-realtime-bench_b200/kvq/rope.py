"""Rotary-embedding tables for the fused rotary + quantize append
(kvq_rope_quantize).

The upstream runtime (Wan's causal model; not vendored in the reference, which
cites its band split at quant_kv.py:26-31) rotates keys with a complex128 table
built once per model: for head_dim 128 the 64 channel pairs split into 22 / 21 /
21 pairs for the frame / height / width axis, pair j of an axis of `dim` real
channels turning at theta^(-2j/dim) radians per position. `freqs` builds that
table the way the upstream does (torch.outer + torch.polar in float64) as
[max_pos, 64, 2] float64 (cos, sin); a model's own table can be passed instead
(torch.view_as_real of its complex128 freqs).
"""
from __future__ import annotations

import torch

ROPE_DIMS = (44, 42, 42)   # real channels per axis for head_dim 128
FRAME_SEQ_LEN = 1560       # tokens per latent frame (30 x 52 patches)
GRID_H, GRID_W = 30, 52


def freqs(max_pos: int = 1024, theta: float = 10000.0, device="cpu") -> torch.Tensor:
    parts = []
    for dim in ROPE_DIMS:
        f = torch.outer(torch.arange(max_pos, dtype=torch.float64),
                        1.0 / torch.pow(theta, torch.arange(0, dim, 2, dtype=torch.float64).div(dim)))
        parts.append(torch.polar(torch.ones_like(f), f))
    return torch.view_as_real(torch.cat(parts, dim=1)).contiguous().to(device)


def grid_positions(t0: int, n: int, device="cpu") -> torch.Tensor:
    """(frame, height, width) int32 [n, 3] of tokens t0 .. t0+n-1 of the latent
    grid (1560 tokens per frame, 30 x 52 patches)."""
    t = torch.arange(t0, t0 + n, dtype=torch.int64)
    return torch.stack([t // FRAME_SEQ_LEN, (t % FRAME_SEQ_LEN) // GRID_W, t % GRID_W], dim=1) \
        .to(torch.int32).contiguous().to(device)
