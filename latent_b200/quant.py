"""Load-time NF4 / per-group INT8 quantization of float factors (torch, any device).

Restates the reference encoders on 32-element row groups so that factors
produced here decode to exactly the values the reference decoders give for
the same bytes:

* NF4 (loader/latent_loader.py:111-130): absmax per group (0 -> 1.0),
  normalise by the fp32 absmax, nearest of the 16 levels with the lowest code
  winning a tie, scale stored as fp16(absmax).
* INT8 (loader/latent_loader.py:148-158): scale = absmax/127 in fp32
  (0 -> 1.0), q = clip(round_half_even(v/scale), -127, 127), fp16 scale.
* Per-group fallback: a group whose NF4 amplitude SNR ||v|| / ||v - nf4(v)||
  (loader/latent_loader.py:173-185) is below 10**(snr_db/20) is stored INT8
  (an all-zero group stays NF4).

The nearest-level search buckets by level midpoints and then compares the
exact fp32 distances of the neighbouring levels, which reproduces numpy's
argmin over all 16 distances.
"""

from __future__ import annotations

from typing import Optional

import torch

from .format import GROUP, GroupedFactor

NF4_LEVELS = (
    -1.0, -0.6961928, -0.52507305, -0.3949175, -0.28444138, -0.18477343, -0.09105004, 0.0,
    0.0795803, 0.1609302, 0.2461123, 0.33791524, 0.44070983, 0.562617, 0.72295684, 1.0,
)


def _levels(device) -> torch.Tensor:
    return torch.tensor(NF4_LEVELS, dtype=torch.float32, device=device)


def nearest_level(norm: torch.Tensor) -> torch.Tensor:
    """Index of the nearest NF4 level for every element (lowest index on ties)."""
    lv = _levels(norm.device)
    mids = (lv[:-1] + lv[1:]) * 0.5
    c = torch.bucketize(norm, mids)
    best = c
    bd = (norm - lv[c]).abs()
    for off in (-1, 1):
        cand = (c + off).clamp(0, 15)
        dd = (norm - lv[cand]).abs()
        better = (dd < bd) | ((dd == bd) & (cand < best))
        best = torch.where(better, cand, best)
        bd = torch.where(better, dd, bd)
    return best.to(torch.uint8)


def _pack(nib: torch.Tensor) -> torch.Tensor:
    """[..., 32] nibbles -> [..., 16] bytes, even element in the low nibble."""
    return (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)


def quantize_factor(values: torch.Tensor, snr_db: Optional[float] = 20.0) -> GroupedFactor:
    """Quantize a [rows, cols] float factor (cols % 32 == 0) to the device layout.

    With ``snr_db=None`` every group is NF4 (the reference's default path).
    """
    if values.dim() != 2 or values.shape[1] % GROUP:
        raise ValueError(f"factor must be [rows, cols] with cols % {GROUP} == 0, got {tuple(values.shape)}")
    rows, cols = values.shape
    g = values.to(torch.float32).reshape(-1, GROUP)
    amax = g.abs().amax(dim=1)
    amax = torch.where(amax == 0, torch.ones_like(amax), amax)
    norm = g / amax[:, None]
    codes = nearest_level(norm)
    scale16 = amax.to(torch.float16)
    lo = _pack(codes)
    hi = torch.zeros_like(lo)
    is_i8 = torch.zeros(g.shape[0], dtype=torch.bool, device=g.device)
    if snr_db is not None:
        deq = _levels(g.device)[codes.long()] * scale16.to(torch.float32)[:, None]
        sig = torch.linalg.vector_norm(g, dim=1)
        noise = torch.linalg.vector_norm(g - deq, dim=1).clamp_min(1e-12)
        is_i8 = ((sig / noise) < torch.tensor(10.0 ** (snr_db / 20.0), dtype=torch.float32)) & (sig > 0)
        if bool(is_i8.any()):
            gi = g[is_i8]
            s = gi.abs().amax(dim=1) / torch.tensor(127.0, dtype=torch.float32, device=g.device)
            s = torch.where(s == 0, torch.ones_like(s), s)
            q = torch.round(gi / s[:, None]).clamp(-127, 127).to(torch.int8)
            u = q.view(torch.uint8)
            lo[is_i8] = _pack(u & 0xF)
            hi[is_i8] = _pack(u >> 4)
            scale16 = scale16.clone()
            scale16[is_i8] = s.to(torch.float16)
    gpr = cols // GROUP
    return GroupedFactor(rows, cols, lo.view(rows, gpr, 16), hi.view(rows, gpr, 16),
                         scale16.view(torch.int16).view(rows, gpr), is_i8.view(rows, gpr))
