"""Device layout of quantized factors (load-time packing).

One factor matrix of one expert, shape [rows, cols] with cols % 32 == 0, is
held as row-aligned 32-element groups:

  lo      uint8 [rows, cols/32, 16]  4-bit codes, two per byte, even element in
                                     the low nibble (loader/latent_loader.py:129)
  hi      uint8 [rows, cols/32, 16]  INT8 groups only: the high nibbles of the
                                     int8 values, same nibble order
  scales  fp16  [rows, cols/32]      NF4: absmax; INT8: absmax/127
  is_int8 bool  [rows, cols/32]

For an NF4 group ``lo`` holds the NF4 codes; for an INT8 group it holds the
low nibbles of the int8 values.  Stacking the experts of one factor kind
gives the ``latent_qmatrix`` of include/latent_ffn.h (codes/scales are the
concatenation, INT8 groups get a bitmap, per-word base counts and a compact
``i8_hi`` table).

On the device every stacked expert matrix is stored in 256-column tile-major
group order: tile c (columns 256c .. 256c+255, narrower for the last tile)
holds its rows one after another, each row its w_c/32 groups of 16 code bytes.
The flat group index q = c*rows*8 + row*(w_c/32) + (col - 256c)/32 addresses
the codes (16 bytes at 16q), the scale (entry q), the INT8 bitmap bit and the
order of the compact high-nibble records.  A matrix of at most 256 columns is
therefore plain row-major.  The order lets a kernel that streams a row range
of one column tile find its codes, scales and INT8 records as three
contiguous runs.

Converters accept the reference's NPZ encodings (loader/latent_loader.py:
NF4 group 32 at :111-145, whole-matrix INT8 group 64 at :148-170) and keep
every decoded value bit-identical: a reference group that spans 64 elements
becomes two 32-element groups carrying the same fp16 scale.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Mapping, Optional, Sequence

import numpy as np
import torch

GROUP = 32
TILE = 256  # columns per device tile
SCALE_ONE = 0x3C00  # fp16 bits of 1.0
ZERO_BYTE = 0x77    # two NF4 codes 7 (= 0.0)


@dataclass
class GroupedFactor:
    """One expert's factor matrix in the row-aligned group layout (torch tensors)."""

    rows: int
    cols: int
    lo: torch.Tensor       # uint8 [rows, cols/32, 16]
    hi: torch.Tensor       # uint8 [rows, cols/32, 16]
    scales: torch.Tensor   # int16 view of fp16 bits [rows, cols/32]
    is_int8: torch.Tensor  # bool [rows, cols/32]

    @property
    def n_int8(self) -> int:
        return int(self.is_int8.sum())

    def to(self, device) -> "GroupedFactor":
        return GroupedFactor(self.rows, self.cols, self.lo.to(device), self.hi.to(device),
                             self.scales.to(device), self.is_int8.to(device))

    def padded(self, rows: int, cols: int) -> "GroupedFactor":
        """Zero-pads to [rows, cols] with NF4 zero groups (code 7, scale 1.0); results are unchanged."""
        if rows < self.rows or cols < self.cols or cols % GROUP:
            raise ValueError(f"cannot pad [{self.rows},{self.cols}] to [{rows},{cols}]")
        if (rows, cols) == (self.rows, self.cols):
            return self
        g = cols // GROUP
        dev = self.lo.device
        lo = torch.full((rows, g, 16), ZERO_BYTE, dtype=torch.uint8, device=dev)
        hi = torch.zeros((rows, g, 16), dtype=torch.uint8, device=dev)
        sc = torch.full((rows, g), SCALE_ONE, dtype=torch.int16, device=dev)
        i8 = torch.zeros((rows, g), dtype=torch.bool, device=dev)
        g0 = self.cols // GROUP
        lo[: self.rows, :g0] = self.lo
        hi[: self.rows, :g0] = self.hi
        sc[: self.rows, :g0] = self.scales
        i8[: self.rows, :g0] = self.is_int8
        return GroupedFactor(rows, cols, lo, hi, sc, i8)


def _shape2(shape: Sequence[int]):
    shape = tuple(int(s) for s in shape)
    if len(shape) != 2:
        raise ValueError(f"factor must be 2-D, got shape {shape}")
    rows, cols = shape
    if cols % GROUP:
        raise ValueError(
            f"factor shape {shape}: the device layout needs the column count to be a multiple of {GROUP} "
            "so every quantization group lies inside one row")
    return rows, cols


def _np_u16(scales) -> np.ndarray:
    a = np.asarray(scales)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    if a.dtype in (np.uint16, np.int16):
        return a.view(np.uint16)
    raise TypeError(f"scales must be fp16, got {a.dtype}")


def from_nf4(packed, scales, shape, group: int = 32) -> GroupedFactor:
    """Reference NF4 arrays (``quantize_nf4`` output, group 32) -> GroupedFactor."""
    if group != GROUP:
        raise ValueError(f"NF4 group size {group} is not supported (the format uses {GROUP})")
    rows, cols = _shape2(shape)
    g = rows * cols // GROUP
    packed = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8).ravel()[: g * 16])
    sc = np.ascontiguousarray(_np_u16(scales).ravel()[:g])
    if packed.size != g * 16 or sc.size != g:
        raise ValueError("NF4 arrays are shorter than the shape requires")
    lo = torch.from_numpy(packed.copy()).view(rows, cols // GROUP, 16)
    return GroupedFactor(rows, cols, lo, torch.zeros_like(lo),
                         torch.from_numpy(sc.view(np.int16).copy()).view(rows, cols // GROUP),
                         torch.zeros((rows, cols // GROUP), dtype=torch.bool))


def _split_int8(q: np.ndarray):
    """int8 values [..., 32] -> (lo nibbles packed [..., 16], hi nibbles packed [..., 16])."""
    u = q.astype(np.int8).view(np.uint8)
    lo_n, hi_n = u & 0xF, u >> 4
    lo = (lo_n[..., 0::2] | (lo_n[..., 1::2] << 4)).astype(np.uint8)
    hi = (hi_n[..., 0::2] | (hi_n[..., 1::2] << 4)).astype(np.uint8)
    return lo, hi


def from_int8(q, scales, shape, group: int = 64) -> GroupedFactor:
    """Reference INT8 arrays (``quantize_int8`` output, group 64 or 32) -> GroupedFactor."""
    rows, cols = _shape2(shape)
    if group % GROUP:
        raise ValueError(f"INT8 group size {group} must be a multiple of {GROUP}")
    g = rows * cols // GROUP
    qv = np.asarray(q, dtype=np.int8).ravel()[: g * GROUP].reshape(g, GROUP)
    sc = _np_u16(scales).ravel()
    sub = group // GROUP
    sc32 = sc[np.arange(g) // sub]
    lo, hi = _split_int8(qv)
    gpr = cols // GROUP
    return GroupedFactor(rows, cols, torch.from_numpy(lo).view(rows, gpr, 16),
                         torch.from_numpy(hi).view(rows, gpr, 16),
                         torch.from_numpy(sc32.view(np.int16).copy()).view(rows, gpr),
                         torch.ones((rows, gpr), dtype=torch.bool))


def from_mixed(nf4, scales, is_int8, int8, shape) -> GroupedFactor:
    """Per-group NF4/INT8 arrays (NF4 codes, per-group scale, INT8 mask, int8 values)."""
    rows, cols = _shape2(shape)
    g = rows * cols // GROUP
    lo = np.asarray(nf4, dtype=np.uint8).ravel()[: g * 16].reshape(g, 16).copy()
    is_i8 = np.asarray(is_int8, dtype=bool).ravel()[:g]
    q = np.asarray(int8, dtype=np.int8).ravel()[: g * GROUP].reshape(g, GROUP)
    lo8, hi8 = _split_int8(q)
    lo[is_i8] = lo8[is_i8]
    hi = np.where(is_i8[:, None], hi8, 0).astype(np.uint8)
    gpr = cols // GROUP
    sc = _np_u16(scales).ravel()[:g]
    return GroupedFactor(rows, cols, torch.from_numpy(lo).view(rows, gpr, 16), torch.from_numpy(hi).view(rows, gpr, 16),
                         torch.from_numpy(sc.view(np.int16).copy()).view(rows, gpr),
                         torch.from_numpy(is_i8.copy()).view(rows, gpr))


def from_npz(arrays: Mapping[str, np.ndarray], name: str, side: str) -> GroupedFactor:
    """One factor from the reference NPZ keys (loader/latent_runtime.py:19-28 order: NF4, then INT8)."""
    shape = tuple(int(v) for v in arrays[f"{name}.{side}.shape"])
    scales = arrays[f"{name}.{side}.scales"]
    if f"{name}.{side}.nf4" in arrays:
        return from_nf4(arrays[f"{name}.{side}.nf4"], scales, shape, 32)
    if f"{name}.{side}.int8" in arrays:
        return from_int8(arrays[f"{name}.{side}.int8"], scales, shape, 64)
    raise KeyError(f"missing {name}.{side} factor")


def tile_order(rows: int, cols: int, device=None) -> torch.Tensor:
    """Row-major group index of each device (tile-major) group position.

    ``tile_order(rows, cols)[q]`` is the row-major group index (row*cols/32 +
    col/32) of flat device group q; see the module docstring.
    """
    gpr = cols // GROUP
    parts = []
    for c0 in range(0, cols, TILE):
        ng = min(TILE, cols - c0) // GROUP
        g0 = c0 // GROUP
        idx = torch.arange(rows, device=device)[:, None] * gpr + g0 + torch.arange(ng, device=device)[None, :]
        parts.append(idx.reshape(-1))
    return torch.cat(parts)


BLOCK_ROWS = 128   # rows of an INT8 list block (one decode stage)
BLOCK_WORDS = 12   # int32 words per block in i8_blocks


def int8_block_lists(is_i8: torch.Tensor, rows: int, cols: int):
    """Per-block INT8 group lists of a stacked factor (the decode kernel's staging tables).

    ``is_i8``: bool [E, g] in device (tile-major) group order.  A block is
    (expert e, 256-column tile c, 128-row block s), index
    b = (e * tiles + c) * row_blocks + s.  ``i8_blocks`` int32 [n_blocks, 12]:
    words 0..8 are the cumulative entry offsets of the block's group columns
    0..7 (column j's entries are [w[j], w[j+1]), w[0] = 0, w[8] = the block's
    INT8 groups), word 9 the index of the block's first entry in ``i8_list``
    (a multiple of 4), word 10 the block's first INT8 record in ``i8_hi``.
    ``i8_list`` uint32 (as int32): one entry per INT8 group, (row in block << 16)
    | (record index - word 10), sorted by column then row, each block's run
    padded to a multiple of 4 entries.
    """
    dev = is_i8.device
    E, g = is_i8.shape
    tiles = (cols + 255) // 256
    rblk = (rows + BLOCK_ROWS - 1) // BLOCK_ROWS
    nb = E * tiles * rblk
    q = torch.arange(g, device=dev)
    c = torch.div(q, rows * 8, rounding_mode="floor")
    within = q - c * rows * 8
    ng = torch.clamp(cols // GROUP - 8 * c, max=8)
    row = torch.div(within, ng, rounding_mode="floor")
    gi = within - row * ng
    blk = c * rblk + torch.div(row, BLOCK_ROWS, rounding_mode="floor")                # per-expert block
    flag = is_i8.reshape(E, g)
    e_idx, q_idx = torch.nonzero(flag, as_tuple=True)                                 # (e, q) order = record order
    rec = torch.arange(e_idx.numel(), device=dev)
    b = e_idx * (tiles * rblk) + blk[q_idx]
    counts = torch.bincount(b, minlength=nb)
    first_rec = torch.cumsum(counts, 0) - counts
    col_counts = torch.bincount(b * 8 + gi[q_idx], minlength=nb * 8).view(nb, 8)
    padded = (counts + 3) // 4 * 4
    blk0 = torch.cumsum(padded, 0) - padded
    words = torch.zeros((nb, BLOCK_WORDS), dtype=torch.int64, device=dev)
    words[:, 1:9] = torch.cumsum(col_counts, 1)
    words[:, 9] = blk0
    words[:, 10] = first_rec
    # entries sorted by (block, column, row); rows within a block are BLOCK_ROWS apart at most
    rib = row[q_idx] % BLOCK_ROWS
    key = (b * 8 + gi[q_idx]) * BLOCK_ROWS + rib
    order = torch.argsort(key)
    b_s = b[order]
    pos = torch.arange(order.numel(), device=dev) - (torch.cumsum(counts, 0) - counts)[b_s]   # rank in block
    entries = torch.zeros(int(padded.sum()) if nb else 0, dtype=torch.int64, device=dev)
    entries[blk0[b_s] + pos] = (rib[order] << 16) | (rec[order] - first_rec[b_s])
    return words.to(torch.int32).contiguous(), entries.to(torch.int32).contiguous()


class StackedFactor:
    """One factor kind of all experts, device-resident, as a ``latent_qmatrix``.

    Tensors (flat group order q of the module docstring): ``codes`` uint8
    [E, g, 16], ``scales`` int16 (fp16 bits) [E, g] with g = rows*cols/32,
    and, when any group is INT8, ``i8_mask`` / ``i8_base`` int32 [E, words]
    (bit q of expert e's mask marks an INT8 group; base = INT8 groups before
    the word over all experts), ``i8_hi`` uint8 [n_int8, 16] in (expert, q)
    order, and the per-block lists ``i8_blocks`` / ``i8_list`` of
    ``int8_block_lists`` (the decode kernel stages these instead of the mask).
    """

    def __init__(self, factors: Sequence[GroupedFactor], device):
        if not factors:
            raise ValueError("no factors to stack")
        rows, cols = factors[0].rows, factors[0].cols
        for f in factors:
            if (f.rows, f.cols) != (rows, cols):
                raise ValueError("all experts of a factor kind must share one (padded) shape")
        self.rows, self.cols, self.n_expert = rows, cols, len(factors)
        dev = torch.device(device)
        E, g = len(factors), rows * cols // GROUP
        perm = tile_order(rows, cols, dev)
        self.codes = torch.stack([f.lo.to(dev).reshape(g, 16) for f in factors])[:, perm].contiguous()
        is_i8 = torch.stack([f.is_int8.to(dev).reshape(g) for f in factors])[:, perm]
        # INT8 groups carry the sign bit of their (non-negative) fp16 scale as a flag.
        sc = torch.stack([f.scales.to(dev).reshape(g) for f in factors])[:, perm]
        sc = torch.where(is_i8, sc | torch.tensor(-0x8000, dtype=torch.int16, device=dev), sc)
        self.scales = sc.contiguous()
        self.int8_per_expert = is_i8.sum(dim=1).cpu().tolist()
        self.n_int8 = int(sum(self.int8_per_expert))
        if self.n_int8:
            words = (g + 31) // 32
            pad = torch.zeros((E, words * 32), dtype=torch.bool, device=dev)
            pad[:, :g] = is_i8
            bits = pad.view(E, words, 32).to(torch.int64) << torch.arange(32, device=dev, dtype=torch.int64)
            w64 = bits.sum(dim=2)
            self.i8_mask = (w64 - (w64 >= 2 ** 31).to(torch.int64) * 2 ** 32).to(torch.int32).contiguous()
            per_word = pad.view(E, words, 32).sum(dim=2).reshape(-1)
            base = torch.cumsum(per_word, 0) - per_word
            self.i8_base = base.to(torch.int32).view(E, words).contiguous()
            hi = torch.stack([f.hi.to(dev).reshape(g, 16) for f in factors])[:, perm].reshape(E * g, 16)
            self.i8_hi = hi[is_i8.reshape(-1)].contiguous()
            self.i8_blocks, self.i8_list = int8_block_lists(is_i8, rows, cols)
            n_blk = self.i8_blocks[:, 8].view(E, -1).to(torch.int64)
            # decode reads a block's 48-byte word row and its padded entries when it has INT8 groups
            self.i8_meta_per_expert = (((n_blk + 3) // 4 * 16 + 48) * (n_blk > 0)).sum(dim=1).cpu().tolist()
        else:
            self.i8_mask = self.i8_base = self.i8_hi = self.i8_blocks = self.i8_list = None

    def nbytes(self, experts: Optional[Sequence[int]] = None) -> int:
        """Bytes the kernels read for the given experts (all when None)."""
        per = self.rows * self.cols // 2 + self.rows * self.cols // GROUP * 2
        n_exp = self.n_expert if experts is None else len(list(experts))
        n = per * n_exp
        if self.n_int8:   # the INT8 list blocks and entries
            n += sum(int(self.i8_meta_per_expert[e]) for e in (range(self.n_expert) if experts is None else experts))
        return n

    def int8_bytes(self, experts: Sequence[int]) -> int:
        """Sidecar bytes (INT8 high nibbles) of the given experts."""
        if not self.n_int8:
            return 0
        return int(sum(int(self.int8_per_expert[e]) for e in experts) * 16)

    def qmatrix(self):
        from ._lib import QMatrix
        ptr = lambda t: None if t is None else t.data_ptr()
        return QMatrix(ptr(self.codes), ptr(self.scales), ptr(self.i8_mask), ptr(self.i8_base), ptr(self.i8_hi),
                       ptr(self.i8_blocks), ptr(self.i8_list), self.rows, self.cols)

    def expert(self, e: int) -> GroupedFactor:
        """Copy of expert ``e`` as a row-major GroupedFactor (host side; for tests and tooling)."""
        g = self.rows * self.cols // GROUP
        perm = tile_order(self.rows, self.cols)
        lo = torch.empty((g, 16), dtype=torch.uint8)
        lo[perm] = self.codes[e].cpu()
        sc = torch.empty(g, dtype=torch.int16)
        sc[perm] = self.scales[e].cpu() & 0x7FFF
        i8 = torch.zeros(g, dtype=torch.bool)
        hi = torch.zeros((g, 16), dtype=torch.uint8)
        if self.n_int8:
            m = self.i8_mask[e].cpu().to(torch.int64) & 0xFFFFFFFF
            bits = ((m[:, None] >> torch.arange(32)) & 1).reshape(-1)[:g].bool()
            first = int(self.i8_base[e, 0])
            n = int(bits.sum())
            hq = torch.zeros((g, 16), dtype=torch.uint8)
            hq[bits] = self.i8_hi[first:first + n].cpu()
            hi[perm] = hq
            i8[perm] = bits
        gpr = self.cols // GROUP
        return GroupedFactor(self.rows, self.cols, lo.view(self.rows, gpr, 16), hi.view(self.rows, gpr, 16),
                             sc.view(self.rows, gpr), i8.view(self.rows, gpr))


KINDS = ("gate_a", "gate_b", "up_a", "up_b", "down_a", "down_b")


class ExpertSet:
    """Device-resident factors of one MoE layer: six stacked factor kinds.

    ``rank`` is the padded rank every expert is stored at (a power of two
    between 32 and 512); experts of lower rank carry zero groups, which do
    not change any result.

    ``dense`` flags dense-fallback experts: ``{expert: {"gate": W_g [d, f],
    "up": W_u [d, f], "down": W_d [f, d]}}`` with any subset of the three
    kinds (the reference's ``<name>.dense_fallback`` copies,
    loader/latent_loader.py:262-265, kept as fp16 on the device).  The routed
    op serves a flagged expert densely: its dense matrices where given, its
    exact factor pairs for the other kinds.
    """

    def __init__(self, experts: Sequence[Mapping[str, GroupedFactor]], device="cuda", rank: Optional[int] = None,
                 dense: Optional[Mapping[int, Mapping[str, object]]] = None):
        if not experts:
            raise ValueError("an ExpertSet needs at least one expert")
        d, r0 = experts[0]["gate_a"].rows, experts[0]["gate_a"].cols
        f = experts[0]["gate_b"].cols
        rmax = max(max(ex["gate_a"].cols, ex["up_a"].cols, ex["down_a"].cols,
                       ex["gate_b"].rows, ex["up_b"].rows, ex["down_b"].rows) for ex in experts)
        if rank is None:
            rank = 32
            while rank < rmax:
                rank *= 2
        if rank < rmax or rank not in (32, 64, 128, 256, 512):
            raise ValueError(f"rank {rank} unsupported for max factor rank {rmax}")
        shapes = {"gate_a": (d, rank), "up_a": (d, rank), "down_a": (f, rank),
                  "gate_b": (rank, f), "up_b": (rank, f), "down_b": (rank, d)}
        for ex in experts:
            for k in KINDS:
                fr = ex[k]
                want = shapes[k]
                if k.endswith("_a") and fr.rows != want[0] or k.endswith("_b") and fr.cols != want[1]:
                    raise ValueError(f"expert factor {k} has shape [{fr.rows},{fr.cols}], expected rows/cols "
                                     f"consistent with {want}")
        self.n_expert, self.n_embd, self.n_ff, self.rank = len(experts), d, f, rank
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.factors = {k: StackedFactor([ex[k].padded(*shapes[k]) for ex in experts], self.device) for k in KINDS}
        dense_shapes = {"gate": (d, f), "up": (d, f), "down": (f, d)}
        self.dense: Dict[int, Dict[str, torch.Tensor]] = {}
        for e, mats in (dense or {}).items():
            e = int(e)
            if not 0 <= e < self.n_expert:
                raise ValueError(f"dense-fallback expert {e} out of range [0, {self.n_expert})")
            kept = {}
            for name, w in mats.items():
                if name not in dense_shapes:
                    raise ValueError(f"unknown dense kind {name!r} (gate, up or down)")
                w = torch.as_tensor(np.asarray(w) if not torch.is_tensor(w) else w)
                if tuple(w.shape) != dense_shapes[name]:
                    raise ValueError(f"dense {name} of expert {e} has shape {tuple(w.shape)}, "
                                     f"expected {dense_shapes[name]}")
                kept[name] = w.to(device=self.device, dtype=torch.float16).contiguous()
            if kept:
                self.dense[e] = kept

    def __getitem__(self, kind: str) -> StackedFactor:
        return self.factors[kind]

    def factor_bytes(self, experts: Sequence[int]) -> int:
        """Algorithmic bytes the kernels stream for the given experts (codes, scales, INT8 tables)."""
        experts = list(experts)
        return sum(self.factors[k].nbytes(experts) + self.factors[k].int8_bytes(experts) for k in KINDS)
