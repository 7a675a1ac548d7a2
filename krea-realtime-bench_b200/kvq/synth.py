"""Seeded synthetic K/V/Q with the shapes and value distributions of the workloads.

No dataset is involved: the reference measures on live model tensors that are not
available, so seeded stand-ins with their statistics are used.
  V ~ N(0, 1)
  K ~ N(0, 1) * exp(sigma * z[h, c]) with z ~ N(0, 1) per (head, channel), i.e.
      log-normal per-channel scales that mimic post-RoPE key outlier channels,
      then a Wan-style 3-axis rotary embedding over (frame, height, width):
      token t -> f = t // 1560, h = (t % 1560) // 52, w = t % 52 (832x480 latents
      with 2x2 patches give 52 x 30 = 1560 tokens per frame); channel pairs
      (2i, 2i+1) rotate by pos * 10000^(-2i/dim) with band widths 44/42/42 real
      channels (quant_kv.py:26-31 describes the bands).
  Q ~ N(0, 1) / sqrt(D)
Values are drawn in fp32 and cast to bf16 once. With device="cpu" the bits are
reproducible everywhere; on CUDA a CUDA generator is used (fast, not
bit-identical to CPU).
"""
from __future__ import annotations

import math

import torch

FRAME_SEQ_LEN = 1560
GRID_W = 52
ROPE_DIMS = (44, 42, 42)  # real channels per rotary band (frame, height, width)


def _gen(seed: int, device) -> torch.Generator:
    dev = torch.device(device)
    g = torch.Generator(device=dev.type if dev.type == "cpu" else dev)
    g.manual_seed(int(seed))
    return g


def rope_cos_sin(positions: torch.Tensor, theta: float = 10000.0):
    """cos/sin [L, 64] (fp32) of the 3-axis rotary embedding for head_dim 128."""
    t = positions.to(torch.int64)
    axes = (t // FRAME_SEQ_LEN, (t % FRAME_SEQ_LEN) // GRID_W, t % GRID_W)
    angles = []
    for pos, dim in zip(axes, ROPE_DIMS):
        inv = theta ** (-torch.arange(0, dim, 2, dtype=torch.float64, device=t.device) / dim)
        angles.append(pos.to(torch.float64)[:, None] * inv[None, :])
    ang = torch.cat(angles, dim=1)  # [L, 64]
    return torch.cos(ang).to(torch.float32), torch.sin(ang).to(torch.float32)


def apply_rope(x: torch.Tensor, pos0: int = 0) -> torch.Tensor:
    """Rotate channel pairs (2i, 2i+1) of x [L, H, 128] (fp32) at positions pos0.."""
    L = x.shape[0]
    cos, sin = rope_cos_sin(torch.arange(pos0, pos0 + L, device=x.device))
    xe, xo = x[..., 0::2], x[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = torch.empty_like(x)
    out[..., 0::2] = xe * c - xo * s
    out[..., 1::2] = xe * s + xo * c
    return out


def make_k(L: int, H: int, D: int = 128, seed: int = 0, pos0: int = 0, sigma: float = 1.0,
           device="cpu") -> torch.Tensor:
    """Post-RoPE keys [L, H, D] bf16 with log-normal channel outliers."""
    g = _gen(seed * 7919 + 11, device)
    base = torch.randn((L, H, D), generator=g, device=device, dtype=torch.float32)
    gz = _gen(seed * 7919 + 13, "cpu")
    chan = torch.exp(sigma * torch.randn((H, D), generator=gz, dtype=torch.float32)).to(device)
    k = base * chan[None]
    if D == 128:
        k = apply_rope(k, pos0)
    return k.to(torch.bfloat16)


def make_v(L: int, H: int, D: int = 128, seed: int = 0, device="cpu") -> torch.Tensor:
    g = _gen(seed * 7919 + 17, device)
    return torch.randn((L, H, D), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


def make_q(B: int, L: int, H: int, D: int = 128, seed: int = 0, device="cpu") -> torch.Tensor:
    g = _gen(seed * 7919 + 19, device)
    q = torch.randn((B, L, H, D), generator=g, device=device, dtype=torch.float32) / math.sqrt(D)
    return q.to(torch.bfloat16)


def make_outlier(L: int, H: int, D: int = 128, seed: int = 0, device="cpu") -> torch.Tensor:
    """The reference kernel test's input style (test_kernels.py:29-33): bf16
    N(0,1)*3 with channel 7 scaled by 40 and channel 60 by 15."""
    g = _gen(seed, device)
    x = torch.randn((L, H, D), generator=g, device=device, dtype=torch.bfloat16) * 3.0
    x[:, :, 7] *= 40
    x[:, :, 60] *= 15
    return x
