"""LATENT GGUF stacked factors -> a device-resident ExpertSet (load time).

The reference writer stores, per MoE layer L (loader/write_latent_gguf.py:
names :72-74, stacking and NF4 packing :126-275, tensor records :412-436):

  blk.L.ffn_latent_{gate,up,down}_{a,b}     I8,  dims (n_expert, rows, cols/2):
        NF4 codes of each row, two per byte, even column in the low nibble,
        rows padded with code 7 (0.0)
  blk.L.ffn_latent_{gate,up,down}_{a,b}_s   F16, dims (n_expert, rows, cols/32):
        the group-32 absmax scales (padding groups 1.0)
  blk.L.ffn_latent_ranks                    I8,  (n_expert, 3): per-expert ranks

with the bytes of each tensor in C order of its recorded dims.  A factors
are [n_in, max_rank] (columns zero-padded to max_rank), B factors
[largest actual rank, n_out].  This reader:

  * reads the codes packed, two per byte, as written (the reference CUDA
    wrapper's strides assume one code per byte, kernels/latent_fused_expert_ffn.cu:199-211);
  * pads A columns and B rows to one power-of-two rank with zero groups,
    which changes no result (zero columns of A meet zero rows of B);
  * does not need the per-expert ranks (their uint8 storage overflows at
    rank >= 256, write_latent_gguf.py:262-265);
  * also accepts the names of the reference's ggml patch
    (``blk.L.ffn_latent_gate_a.weight`` / ``.scales``), which differ from the
    writer's.

Missing tensors raise ``KeyError`` (as ``load_pair`` does for NPZ keys).
The GGUF container itself is parsed by the ``gguf`` package.
"""

from __future__ import annotations

from pathlib import Path
from typing import Dict, Optional, Tuple

import numpy as np

from .format import ExpertSet, from_nf4

KINDS = ("gate", "up", "down")
SIDES = ("a", "b")


def _tensor(tensors: Dict[str, object], names) -> np.ndarray:
    for n in names:
        t = tensors.get(n)
        if t is not None:
            dims = tuple(int(x) for x in t.shape)
            return np.asarray(t.data).reshape(-1).view(np.uint8 if t.data.dtype == np.int8 else t.data.dtype) \
                .reshape(dims)
    raise KeyError(f"none of {list(names)} in the GGUF")


def read_layer(path, layer: int) -> Dict[Tuple[str, str], Tuple[np.ndarray, np.ndarray]]:
    """{(kind, side): (codes uint8 [E, rows, cols/2], scales fp16 [E, rows, cols/32])} of one layer."""
    from gguf import GGUFReader
    reader = GGUFReader(str(Path(path)))
    tensors = {t.name: t for t in reader.tensors}
    out = {}
    for kind in KINDS:
        for side in SIDES:
            base = f"blk.{layer}.ffn_latent_{kind}_{side}"
            codes = _tensor(tensors, (base, base + ".weight"))
            scales = _tensor(tensors, (base + "_s", base + ".scales"))
            if scales.dtype != np.float16:
                raise ValueError(f"{base}: scales must be F16, got {scales.dtype}")
            if codes.ndim != 3 or scales.ndim != 3 or codes.shape[:2] != scales.shape[:2] or \
                    codes.shape[2] * 2 != scales.shape[2] * 32:
                raise ValueError(f"{base}: codes {codes.shape} and scales {scales.shape} do not describe "
                                 "group-32 NF4 rows")
            out[(kind, side)] = (codes, scales)
    n_e = {v[0].shape[0] for v in out.values()}
    if len(n_e) != 1:
        raise ValueError(f"layer {layer}: factor tensors disagree on the expert count {sorted(n_e)}")
    return out


def load_layer(path, layer: int, device="cuda", rank: Optional[int] = None) -> ExpertSet:
    """One MoE layer of a LATENT GGUF as an ExpertSet on ``device`` (ready for ExpertFFN)."""
    raw = read_layer(path, layer)
    n_expert = next(iter(raw.values()))[0].shape[0]
    experts = []
    for e in range(n_expert):
        facs = {}
        for (kind, side), (codes, scales) in raw.items():
            rows, half = codes.shape[1], codes.shape[2]
            facs[f"{kind}_{side}"] = from_nf4(codes[e].reshape(-1), scales[e].reshape(-1), (rows, 2 * half))
        experts.append(facs)
    return ExpertSet(experts, device=device, rank=rank)
