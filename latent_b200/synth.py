"""Seeded synthetic MoE layers with the shapes and statistics of the benchmark configs.

Recipe (per expert, per matrix W of shape [n_in, n_out]):
  W = U diag(s) V^T + N(0, noise^2),  U, V Haar-orthogonal (QR of a Gaussian
  with the sign of diag(R) folded in), s_i = 0.5 * i^-0.8;
  rank-r truncation A = U_r sqrt(S_r), B = sqrt(S_r) V_r^T (the reference's
  make_factors, loader/latent_loader.py:104-108) from a randomized SVD with
  oversampling 16 and one power iteration (the reference's randomized_svd,
  :66-90); then NF4 group-32 quantization with per-group INT8 fallback below
  20 dB (``latent_b200.quant``).
  ``exact=False`` skips the noise and the SVD and takes the factors straight
  from a rank-r construction -- the exact top-r SVD of the noiseless W --
  which is what large configs use to keep generation to seconds.
Routing: logits ~ N(0,1) [T, E] (+ a Zipf(a) per-expert bias when asked),
softmax, top-k, weights renormalised to sum to 1.  x ~ N(0,1) in the
config's activation dtype.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .format import ExpertSet, GroupedFactor
from .quant import quantize_factor


@dataclass(frozen=True)
class LayerConfig:
    name: str
    n_expert: int
    n_embd: int
    n_ff: int
    rank: int
    top_k: int
    n_tokens: int
    x_dtype: torch.dtype = torch.bfloat16
    snr_db: Optional[float] = 20.0
    outlier_frac: float = 0.0    # fraction of columns of W scaled x20 before the SVD
    zipf: Optional[float] = None  # per-expert router bias exponent
    exact: bool = True
    noise: float = 1e-4
    seed: int = 0


CONFIGS: Dict[int, LayerConfig] = {
    0: LayerConfig("c0-toy", 8, 1024, 704, 128, 2, 64, torch.float32, seed=0),
    1: LayerConfig("c1-v2lite-decode", 64, 2048, 1408, 256, 6, 32, torch.bfloat16, seed=1),
    2: LayerConfig("c2-mixtral-prefill", 8, 4096, 14336, 512, 2, 8192, torch.bfloat16, outlier_frac=0.04, seed=2),
    3: LayerConfig("c3-v3-prefill", 256, 7168, 2048, 256, 8, 16384, torch.bfloat16, zipf=1.1, exact=False, seed=3),
    4: LayerConfig("c4-v3-decode", 256, 7168, 2048, 256, 8, 64, torch.bfloat16, exact=False, seed=4),
}


def sweep_config(rank: int, batch: int) -> LayerConfig:
    """One point of the c4 decode sweep (rank in {64,128,256,512}, batch in {1,8,64,256})."""
    return replace(CONFIGS[4], name=f"c4-v3-decode-r{rank}-b{batch}", rank=rank, n_tokens=batch)


def _haar(m: int, k: int, gen: torch.Generator, device) -> torch.Tensor:
    q, r = torch.linalg.qr(torch.randn((m, k), generator=gen, device=device, dtype=torch.float32))
    return q * torch.sign(torch.diagonal(r))[None, :]


def _rsvd(w: torch.Tensor, rank: int, gen: torch.Generator, oversample: int = 16, power: int = 1):
    m, n = w.shape
    k = min(rank + oversample, m, n)
    omega = torch.randn((n, k), generator=gen, device=w.device, dtype=torch.float32)
    y = w @ omega
    for _ in range(power):
        y = w @ (w.T @ y)
    q, _ = torch.linalg.qr(y)
    u_hat, s, vt = torch.linalg.svd(q.T @ w, full_matrices=False)
    return (q @ u_hat)[:, :rank], s[:rank], vt[:rank]


def spectral_factors(n_in: int, n_out: int, rank: int, gen: torch.Generator, device, exact: bool = True,
                     noise: float = 1e-4, outlier_frac: float = 0.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Float factors A [n_in, rank], B [rank, n_out] of one synthetic expert matrix."""
    if not exact:
        s = 0.5 * torch.arange(1, rank + 1, device=device, dtype=torch.float32) ** -0.8
        u, v = _haar(n_in, rank, gen, device), _haar(n_out, rank, gen, device)
        root = s.sqrt()
        return u * root[None, :], root[:, None] * v.T
    k = min(n_in, n_out)
    s = 0.5 * torch.arange(1, k + 1, device=device, dtype=torch.float32) ** -0.8
    u, v = _haar(n_in, k, gen, device), _haar(n_out, k, gen, device)
    w = (u * s[None, :]) @ v.T
    if noise:
        w = w + noise * torch.randn((n_in, n_out), generator=gen, device=device, dtype=torch.float32)
    if outlier_frac > 0:
        n_cols = max(1, int(round(outlier_frac * n_out)))
        cols = torch.randperm(n_out, generator=gen, device=device)[:n_cols]
        w[:, cols] *= 20.0
    ur, sr, vtr = _rsvd(w, rank, gen)
    root = sr.clamp_min(0).sqrt()
    return ur * root[None, :], root[:, None] * vtr


def make_expert_factors(cfg: LayerConfig, device="cpu", experts: Optional[Sequence[int]] = None
                        ) -> List[Dict[str, GroupedFactor]]:
    """Quantized factors of the config's experts (all, or the listed ones), on ``device``."""
    out = []
    ids = range(cfg.n_expert) if experts is None else experts
    for e in ids:
        gen = torch.Generator(device=device)
        gen.manual_seed(1_000_003 * cfg.seed + 7919 * e + 17)
        ex = {}
        for name, (n_in, n_out) in (("gate", (cfg.n_embd, cfg.n_ff)), ("up", (cfg.n_embd, cfg.n_ff)),
                                    ("down", (cfg.n_ff, cfg.n_embd))):
            a, b = spectral_factors(n_in, n_out, cfg.rank, gen, device, cfg.exact, cfg.noise, cfg.outlier_frac)
            ex[f"{name}_a"] = quantize_factor(a, cfg.snr_db)
            ex[f"{name}_b"] = quantize_factor(b, cfg.snr_db)
        out.append(ex)
    return out


def make_expert_set(cfg: LayerConfig, device="cuda", gen_device=None) -> ExpertSet:
    gen_device = device if gen_device is None else gen_device
    return ExpertSet(make_expert_factors(cfg, gen_device), device=device, rank=cfg.rank)


def make_batch(cfg: LayerConfig, device="cpu", n_tokens: Optional[int] = None, seed_offset: int = 0):
    """(x [T, d], ids int32 [T, k], weights fp32 [T, k]) for the config's router recipe."""
    T = cfg.n_tokens if n_tokens is None else n_tokens
    gen = torch.Generator(device=device)
    gen.manual_seed(7_777_777 * (cfg.seed + 1) + 31 * seed_offset)
    x = torch.randn((T, cfg.n_embd), generator=gen, device=device, dtype=torch.float32).to(cfg.x_dtype)
    logits = torch.randn((T, cfg.n_expert), generator=gen, device=device, dtype=torch.float32)
    if cfg.zipf is not None:
        perm = torch.randperm(cfg.n_expert, generator=gen, device=device)
        rank = perm.to(torch.float32) + 1.0
        logits = logits + (-cfg.zipf) * torch.log(rank)[None, :]
    probs = torch.softmax(logits, dim=1)
    w, ids = torch.topk(probs, cfg.top_k, dim=1)
    w = w / w.sum(dim=1, keepdim=True)
    return x.contiguous(), ids.to(torch.int32).contiguous(), w.to(torch.float32).contiguous()
