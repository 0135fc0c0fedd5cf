"""Load-time compression of dense expert matrices on the GPU.

The reference compressor (loader/latent_loader.py:66-108, 173-280,
``compress_matrix``) runs on the host in numpy.  This module runs its stages
on the device:

1. rank: ``choose_rank`` on the full singular values (energy rule of
   latent_loader.py:93-101), singular values by cuSOLVER;
2. ``randomized_svd`` (latent_loader.py:66-90) with the same seeded Gaussian
   test matrix (numpy ``default_rng(seed).standard_normal``, float32),
   oversampling 16 and one power iteration, products and factorizations by
   cuBLAS / cuSOLVER in fp32 (TF32 off);
3. ``make_factors`` A = U sqrt(S), B = sqrt(S) Vt (latent_loader.py:104-108);
4. quantisation by the library kernel ``latent_quantize_groups``: the
   reference NF4 encoder per 32-element row group, and, where a group's NF4
   amplitude SNR is below ``snr_db``, the group in INT8 (the device format's
   per-group fallback, in place of the reference's whole-pair INT8 g64);
5. the dense fp16 fallback copy when the quantised relative error exceeds
   ``error_threshold`` (latent_loader.py:262-265); the routed op serves it
   through ``ExpertSet(dense=...)``.

The rank is padded with zero columns of A / rows of B to a multiple of 32
(the row-group format), which changes no product.  The SVD stages agree with
the reference to fp32 rounding, not bitwise (different LAPACK/cuSOLVER
algorithms); the quantisation of given factors is byte-exact.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional

import numpy as np
import torch

from . import _lib
from .format import GROUP, GroupedFactor

__all__ = ["choose_rank", "randomized_svd", "quantize_groups", "compress_matrix", "CompressedMatrix"]


def choose_rank(singular_values: torch.Tensor, energy: float, min_rank: int, max_rank: int) -> int:
    """Smallest rank whose cumulative energy reaches ``energy`` (latent_loader.py:93-101)."""
    if not 0 < energy <= 1:
        raise ValueError("energy must be in (0, 1]")
    s2 = singular_values.double() ** 2
    total = float(s2.sum())
    if total == 0:
        return min_rank
    cumulative = torch.cumsum(s2, 0) / total
    rank = int(torch.searchsorted(cumulative, torch.tensor([energy], dtype=torch.float64,
                                                           device=cumulative.device)).item()) + 1
    return max(min_rank, min(rank, max_rank, singular_values.numel()))


def randomized_svd(matrix: torch.Tensor, target_rank: int, oversample: int = 16, power_iterations: int = 1,
                   seed: int = 0):
    """Truncated randomized SVD with the reference's test matrix (latent_loader.py:66-90)."""
    m, n = matrix.shape
    rank = min(target_rank, m, n)
    sketch = min(rank + oversample, m, n)
    omega = np.random.default_rng(seed).standard_normal((n, sketch), dtype=np.float32)
    omega = torch.from_numpy(omega).to(matrix.device)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        y = matrix @ omega
        for _ in range(power_iterations):
            y = matrix @ (matrix.T @ y)
        q, _ = torch.linalg.qr(y, mode="reduced")
        b = q.T @ matrix
        u_hat, s, vt = torch.linalg.svd(b, full_matrices=False)
        u = q @ u_hat
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return u[:, :rank], s[:rank], vt[:rank, :]


def quantize_groups(values: torch.Tensor, snr_db: Optional[float] = 20.0):
    """[rows, cols] fp32 CUDA tensor (cols % 32 == 0) -> (GroupedFactor, per-group NF4 SNR) by the kernel."""
    if not values.is_cuda:
        raise ValueError("quantize_groups runs on the GPU (no CPU fallback)")
    if values.dim() != 2 or values.shape[1] % GROUP:
        raise ValueError(f"factor must be [rows, cols] with cols % {GROUP} == 0, got {tuple(values.shape)}")
    rows, cols = values.shape
    v = values.to(torch.float32).contiguous()
    g = rows * cols // GROUP
    dev = v.device
    lo = torch.empty((g, 16), dtype=torch.uint8, device=dev)
    hi = torch.empty((g, 16), dtype=torch.uint8, device=dev)
    sc = torch.empty(g, dtype=torch.int16, device=dev)
    i8 = torch.empty(g, dtype=torch.uint8, device=dev)
    snr = torch.empty(g, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().latent_quantize_groups(
        v.data_ptr(), g, float("nan") if snr_db is None else float(snr_db), lo.data_ptr(), hi.data_ptr(),
        sc.data_ptr(), i8.data_ptr(), snr.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
        "latent_quantize_groups")
    gpr = cols // GROUP
    gf = GroupedFactor(rows, cols, lo.view(rows, gpr, 16), hi.view(rows, gpr, 16), sc.view(rows, gpr),
                       i8.bool().view(rows, gpr))
    return gf, snr


@dataclass
class CompressedMatrix:
    a: GroupedFactor                    # [m, rank padded to 32]
    b: GroupedFactor                    # [rank padded to 32, n]
    rank: int
    report: Dict[str, float] = field(default_factory=dict)
    dense: Optional[torch.Tensor] = None   # fp16 dense fallback copy
    a_float: Optional[torch.Tensor] = None  # the unquantised factors [m, rank], [rank, n]
    b_float: Optional[torch.Tensor] = None


def _rel(ref: torch.Tensor, cand: torch.Tensor) -> float:
    den = float(torch.linalg.norm(ref.double()))
    return 0.0 if den == 0 else float(torch.linalg.norm((ref - cand).double()) / den)


def compress_matrix(matrix, energy: float = 0.99, min_rank: int = 8, max_rank: int = 512,
                    snr_db: Optional[float] = 20.0, error_threshold: float = 0.35, seed: int = 0,
                    device=None) -> CompressedMatrix:
    """One dense matrix -> quantised low-rank pair on the GPU (the stages of latent_loader.py:195-280)."""
    from .runtime import _device, dequantize
    dev = _device(device if device is not None else (matrix.device if torch.is_tensor(matrix) and matrix.is_cuda
                                                     else None))
    w = torch.as_tensor(np.asarray(matrix, dtype=np.float32) if not torch.is_tensor(matrix) else matrix)
    w = w.to(device=dev, dtype=torch.float32).contiguous()
    if w.dim() != 2:
        raise ValueError(f"expected a 2D matrix, got {tuple(w.shape)}")
    full_s = torch.linalg.svdvals(w)
    rank = choose_rank(full_s, energy, min_rank, max_rank)
    u, s, vt = randomized_svd(w, rank, seed=seed)
    root = s[:rank].clamp_min(0).sqrt()
    a = u[:, :rank] * root[None, :]
    b = root[:, None] * vt[:rank, :]
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        dense_error = _rel(w, a @ b)
        rp = -(-rank // GROUP) * GROUP
        a_p = torch.nn.functional.pad(a, (0, rp - rank))
        b_p = torch.nn.functional.pad(b, (0, 0, 0, rp - rank))
        if b_p.shape[1] % GROUP:
            raise ValueError(f"n = {b_p.shape[1]} must be a multiple of {GROUP}")
        qa, snr_a = quantize_groups(a_p, snr_db)
        qb, snr_b = quantize_groups(b_p, snr_db)
        quant_error = _rel(w, dequantize(qa) @ dequantize(qb))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    # the NF4 SNR of the groups holding factor values (B's padding rows excluded)
    real = torch.cat([snr_a, snr_b[: rank * (b_p.shape[1] // GROUP)]])
    thr = 10.0 ** ((snr_db if snr_db is not None else 20.0) / 20.0)
    report = {
        "rank": float(rank),
        "retained_energy": float((s[:rank].double() ** 2).sum() / (full_s.double() ** 2).sum()),
        "dense_relative_error": dense_error,
        "quantized_relative_error": quant_error,
        "min_group_snr": float(real.min()) if real.numel() else float("inf"),
        "low_snr_group_fraction": float((real < thr).float().mean()) if real.numel() else 0.0,
        "int8_groups": float(qa.is_int8.sum() + qb.is_int8.sum()),
    }
    out = CompressedMatrix(qa, qb, rank, report, a_float=a, b_float=b)
    if quant_error > error_threshold:
        out.dense = w.to(torch.float16)
        report["dense_fallback"] = 1.0
    return out
