"""Helpers shared by the GPU parity tests: oracle views of device-format experts."""

import numpy as np
import torch

import oracle as O
from latent_b200 import format as F


def decode(gf: F.GroupedFactor) -> np.ndarray:
    return O.decode_grouped(gf.lo.cpu().numpy(), gf.hi.cpu().numpy(), gf.scales.cpu().numpy().view(np.uint16),
                            gf.is_int8.cpu().numpy(), gf.rows, gf.cols)


def oracle_experts(expert_factors, rank=None):
    """[(gate, up, down)] fp32 (A, B) pairs decoded by the oracle, zero-padded to ``rank``."""
    out = []
    for ex in expert_factors:
        pairs = []
        for name in ("gate", "up", "down"):
            a, b = ex[f"{name}_a"], ex[f"{name}_b"]
            if rank is not None:
                a, b = a.padded(a.rows, rank), b.padded(rank, b.cols)
            pairs.append((decode(a), decode(b)))
        out.append(tuple(pairs))
    return out


def golden_moe_experts(z):
    E = int(z["E"])
    facs, ref = [], []
    for e in range(E):
        arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(f"e{e}/")}
        facs.append({f"{n}_{s}": F.from_npz(arrays, n, s) for n in ("gate", "up", "down") for s in ("a", "b")})
        ref.append(tuple(O.pair_from_npz(arrays, n) for n in ("gate", "up", "down")))
    return facs, ref


def rel(ref, got) -> float:
    if torch.is_tensor(got):
        got = got.detach().cpu().numpy()
    return O.rel_l2(ref, got)
