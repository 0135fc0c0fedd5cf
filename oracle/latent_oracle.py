"""CPU restatement of LATENT's latent expert FFN path (numpy).

TEST INFRASTRUCTURE ONLY -- the checker for the CUDA library and the timed
CPU baseline in ``bench.py``.  The product package never imports it.

Each function names the reference code (paths inside the Yxmura/latent
checkout) whose behaviour it restates.  The reference is plain numpy, so the
restatement keeps the same arithmetic: fp32 values, one fp32 multiply per
dequantized element, fp32 GEMMs, a float64 SiLU rounded to fp32.

Extension beyond the reference (documented, not invented semantics): a
*per-group* NF4/INT8 mix.  The reference falls back to INT8 for a whole A/B
pair (loader/latent_loader.py:229-249); the benchmark recipe asks for a
per-group fallback ("any group with SNR below 20 dB falls back to INT8").
``mixed_encode`` applies the reference's own SNR definition
(loader/latent_loader.py:173-185) and the reference's own INT8 encoder
(:148-158) to single 32-element groups.
"""

from __future__ import annotations

import math
from typing import Dict, List, Mapping, Sequence, Tuple

import numpy as np

__all__ = [
    "adaptive_keep",
    "router_topk",
    "NF4_LEVELS",
    "nf4_encode",
    "nf4_decode",
    "int8_encode",
    "int8_decode",
    "group_snr",
    "mixed_encode",
    "mixed_decode",
    "decode_grouped",
    "silu",
    "project",
    "swiglu_expert",
    "dense_swiglu_expert",
    "factor_from_npz",
    "pair_from_npz",
    "route",
    "moe_forward",
    "rel_l2",
]

# The 16 NF4 levels, in code order.  The values have to be the reference's
# exactly (loader/latent_loader.py:28-48): code 7 is 0.0 and code 15 is 1.0.
NF4_LEVELS = np.array(
    [-1.0, -0.6961928, -0.52507305, -0.3949175, -0.28444138, -0.18477343,
     -0.09105004, 0.0, 0.0795803, 0.1609302, 0.2461123, 0.33791524,
     0.44070983, 0.562617, 0.72295684, 1.0],
    dtype=np.float32,
)


def _grouped(values: np.ndarray, group: int) -> Tuple[np.ndarray, int]:
    flat = np.asarray(values, dtype=np.float32).ravel()
    n_groups = -(-flat.size // group)
    buf = np.zeros(n_groups * group, dtype=np.float32)
    buf[: flat.size] = flat
    return buf.reshape(n_groups, group), flat.size


def nf4_encode(values: np.ndarray, group: int = 32):
    """NF4 encoder: loader/latent_loader.py:111-130.

    Per group of ``group`` flat elements: absmax (0 -> 1.0), normalise by the
    fp32 absmax, nearest level (lowest code on a tie), two codes per byte with
    the even element in the low nibble, code 7 pads an odd count; the scale is
    stored as fp16(absmax).
    """
    g, _ = _grouped(values, group)
    amax = np.abs(g).max(axis=1)
    amax[amax == 0] = np.float32(1.0)
    norm = g / amax[:, None]
    # nearest level; np.argmin keeps the first (lowest) code on exact ties
    codes = np.abs(norm[:, :, None] - NF4_LEVELS[None, None, :]).argmin(axis=2)
    codes = codes.astype(np.uint8).ravel()
    if codes.size & 1:
        codes = np.append(codes, np.uint8(7))
    packed = (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8)
    return packed, amax.astype(np.float16), tuple(np.shape(values))


def nf4_decode(packed: np.ndarray, scales: np.ndarray, shape: Sequence[int], group: int = 32) -> np.ndarray:
    """NF4 decoder: loader/latent_loader.py:133-145.

    value = level[code] * float32(fp16 scale) -- one fp32 rounding.
    """
    packed = np.asarray(packed, dtype=np.uint8).ravel()
    codes = np.stack([packed & 0xF, packed >> 4], axis=1).ravel()
    n = int(np.prod(shape))
    n_groups = -(-n // group)
    codes = codes[: n_groups * group].reshape(n_groups, group)
    vals = NF4_LEVELS[codes] * np.asarray(scales).astype(np.float32)[:, None]
    return vals.ravel()[:n].reshape(tuple(shape)).astype(np.float32)


def int8_encode(values: np.ndarray, group: int = 64):
    """Symmetric INT8 encoder: loader/latent_loader.py:148-158.

    scale = absmax/127 in fp32 (0 -> 1.0); q = clip(rint(v/scale), -127, 127);
    the scale is stored as fp16.
    """
    g, _ = _grouped(values, group)
    scale = np.abs(g).max(axis=1) / np.float32(127.0)
    scale[scale == 0] = np.float32(1.0)
    q = np.clip(np.rint(g / scale[:, None]), -127, 127).astype(np.int8)
    return q.ravel(), scale.astype(np.float16), tuple(np.shape(values))


def int8_decode(q: np.ndarray, scales: np.ndarray, shape: Sequence[int], group: int = 64) -> np.ndarray:
    """INT8 decoder: loader/latent_loader.py:161-170 (float32(q) * float32(scale))."""
    n = int(np.prod(shape))
    n_groups = -(-n // group)
    qg = np.asarray(q, dtype=np.int8).ravel()[: n_groups * group].reshape(n_groups, group)
    vals = qg.astype(np.float32) * np.asarray(scales).astype(np.float32)[:, None]
    return vals.ravel()[:n].reshape(tuple(shape)).astype(np.float32)


def group_snr(ref: np.ndarray, cand: np.ndarray, group: int) -> np.ndarray:
    """Per-group amplitude SNR ||ref|| / max(||ref - cand||, 1e-12): loader/latent_loader.py:173-185."""
    r, _ = _grouped(ref, group)
    c, _ = _grouped(cand, group)
    sig = np.linalg.norm(r, axis=1)
    noise = np.linalg.norm(r - c, axis=1)
    return sig / np.maximum(noise, 1e-12)


def mixed_encode(values: np.ndarray, snr_db: float = 20.0, group: int = 32) -> Dict[str, np.ndarray]:
    """Per-group NF4 with INT8 fallback (the benchmark recipe's extension).

    Every ``group``-element group is NF4-encoded; a group whose amplitude SNR
    (reference definition) is below ``10**(snr_db/20)`` is re-encoded with the
    reference INT8 encoder applied to that group alone (an all-zero group, SNR
    0 by that definition, stays NF4).  Returns the NF4 codes
    (packed), one fp16 scale per group (NF4 absmax or INT8 absmax/127), a bool
    mask of INT8 groups and the int8 values of every group (zeros for NF4
    groups).
    """
    shape = tuple(np.shape(values))
    packed, scales, _ = nf4_encode(values, group)
    deq = nf4_decode(packed, scales, shape, group)
    snr = group_snr(values, deq, group)
    g, _ = _grouped(values, group)
    is_i8 = (snr < np.float32(10.0 ** (snr_db / 20.0))) & np.any(g != 0, axis=1)   # an all-zero group stays NF4
    q_all = np.zeros_like(g, dtype=np.int8)
    scales = scales.copy()
    if is_i8.any():
        q, s, _ = int8_encode(g[is_i8], group)
        q_all[is_i8] = q.reshape(-1, group)
        scales[is_i8] = s
    return {"nf4": packed, "scales": scales, "is_int8": is_i8, "int8": q_all.ravel(), "shape": np.array(shape)}


def mixed_decode(enc: Mapping[str, np.ndarray], group: int = 32) -> np.ndarray:
    shape = tuple(int(s) for s in enc["shape"])
    out = nf4_decode(enc["nf4"], enc["scales"], shape, group).ravel()
    n = out.size
    is_i8 = np.asarray(enc["is_int8"], dtype=bool)
    if is_i8.any():
        i8 = int8_decode(enc["int8"], enc["scales"], (is_i8.size * group,), group).reshape(-1, group)
        full = np.zeros(is_i8.size * group, dtype=np.float32)
        full[:n] = out
        full = full.reshape(-1, group)
        full[is_i8] = i8[is_i8]
        out = full.ravel()[:n]
    return out.reshape(shape)


def decode_grouped(lo: np.ndarray, hi: np.ndarray, scales: np.ndarray, is_int8: np.ndarray,
                   rows: int, cols: int) -> np.ndarray:
    """Decode the row-aligned group layout the CUDA library consumes.

    ``lo``/``hi`` are [groups, 16] packed nibbles, ``scales`` fp16 (or its bit
    pattern) [groups], ``is_int8`` bool [groups].  NF4 groups go through the
    reference NF4 decoder (loader/latent_loader.py:133-145) with their codes
    in ``lo``; INT8 groups through the reference INT8 decoder (:161-170) with
    q = int8(hi << 4 | lo).
    """
    lo = np.asarray(lo, dtype=np.uint8).reshape(-1, 16)
    hi = np.asarray(hi, dtype=np.uint8).reshape(-1, 16)
    sc = np.asarray(scales).reshape(-1)
    sc = sc.view(np.float16) if sc.dtype != np.float16 else sc
    is_i8 = np.asarray(is_int8, dtype=bool).reshape(-1)
    n_groups = lo.shape[0]
    out = nf4_decode(lo.ravel(), sc, (n_groups * 32,), 32).reshape(n_groups, 32)
    if is_i8.any():
        def nib(b):
            return np.stack([b & 0xF, b >> 4], axis=-1).reshape(b.shape[0], 32)
        q = ((nib(hi[is_i8]) << 4) | nib(lo[is_i8])).astype(np.uint8).view(np.int8)
        out[is_i8] = int8_decode(q.ravel(), sc[is_i8], (int(is_i8.sum()) * 32,), 32).reshape(-1, 32)
    return out.reshape(rows, cols)


def silu(x: np.ndarray) -> np.ndarray:
    """SiLU evaluated in float64, clipped to +-1e30, rounded to fp32: loader/latent_runtime.py:39-45."""
    d = np.asarray(x, dtype=np.float32).astype(np.float64)
    return np.clip(d / (1.0 + np.exp(-d)), -1e30, 1e30).astype(np.float32)


def project(x: np.ndarray, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """(x @ A) @ B in fp32: loader/latent_runtime.py:35-36."""
    return (np.asarray(x, dtype=np.float32) @ a) @ b


def swiglu_expert(x, gate, up, down, weight=1.0, weight_before_down=False) -> np.ndarray:
    """SwiGLU over factor pairs: loader/latent_runtime.py:48-59.

    ``gate``/``up``/``down`` are (A, B) fp32 tuples.  ``weight`` may be a
    scalar or a per-row vector; it only enters when ``weight_before_down``.
    """
    h = silu(project(x, *gate)) * project(x, *up)
    if weight_before_down:
        w = np.asarray(weight, dtype=np.float32)
        h = h * (w[:, None] if w.ndim == 1 else w)
    return project(h, *down)


def dense_swiglu_expert(x, gate, up, down, weight=1.0, weight_before_down=False) -> np.ndarray:
    """Dense SwiGLU reference: loader/latent_runtime.py:62-73."""
    x32 = np.asarray(x, dtype=np.float32)
    h = silu(x32 @ gate) * (x32 @ up)
    if weight_before_down:
        w = np.asarray(weight, dtype=np.float32)
        h = h * (w[:, None] if w.ndim == 1 else w)
    return h @ down


def factor_from_npz(arrays: Mapping[str, np.ndarray], name: str, side: str) -> np.ndarray:
    """One factor from reference NPZ keys: loader/latent_runtime.py:19-28 (NF4 g32 first, then INT8 g64)."""
    shape = tuple(int(v) for v in arrays[f"{name}.{side}.shape"])
    scales = arrays[f"{name}.{side}.scales"]
    if f"{name}.{side}.nf4" in arrays:
        return nf4_decode(arrays[f"{name}.{side}.nf4"], scales, shape, 32)
    if f"{name}.{side}.int8" in arrays:
        return int8_decode(arrays[f"{name}.{side}.int8"], scales, shape, 64)
    raise KeyError(f"missing {name}.{side} factor")


def pair_from_npz(arrays: Mapping[str, np.ndarray], name: str) -> Tuple[np.ndarray, np.ndarray]:
    """loader/latent_runtime.py:31-32."""
    return factor_from_npz(arrays, name, "a"), factor_from_npz(arrays, name, "b")


def route(ids: np.ndarray, n_expert: int):
    """Stable grouping of routed (token, slot) pairs by expert.

    Returns (counts[E], offsets[E+1], order) where ``order`` lists flat slot
    indices t*k+j with id >= 0, sorted by expert and, within an expert, by
    slot index.  Slots with id < 0 are skipped (the reference op writes a
    zero row for them: kernels/latent_fused_expert_ffn.cu:33-40).
    """
    flat = np.asarray(ids, dtype=np.int64).ravel()
    valid = np.nonzero(flat >= 0)[0]
    order = valid[np.argsort(flat[valid], kind="stable")]
    counts = np.bincount(flat[valid], minlength=n_expert)[:n_expert]
    offsets = np.concatenate([[0], np.cumsum(counts)])
    return counts, offsets, order


def moe_forward(
    x: np.ndarray,
    ids: np.ndarray,
    weights: np.ndarray,
    experts: Sequence[Tuple[Tuple[np.ndarray, np.ndarray], ...]],
    weight_before_down: bool = False,
    out_per_slot: bool = False,
) -> np.ndarray:
    """Routed expert FFN + top-k combine (the GGML_OP_LATENT_EXPERT_FFN semantics).

    ``experts[e] = (gate, up, down)`` with fp32 (A, B) pairs.  Per routed slot
    the expert output is swiglu_expert(x[t], ...) (latent_runtime.py:48-59);
    ids < 0 contribute zero (kernels/latent_fused_expert_ffn.cu:33-40).
    ``out_per_slot`` returns [T, k, d] per-slot rows like the op's dst
    (kernels/latent_fused_expert_ffn.cu:259, 281-286; weighted only when
    ``weight_before_down``); otherwise out[t] = sum_j w[t,j] * y_j (or the
    plain sum when the weight was applied before the down projection),
    accumulated in float64 in slot order (README.md:108-113,
    kernels/latent_fused_expert_ffn.cu:122-132).
    """
    x32 = np.asarray(x, dtype=np.float32)
    ids = np.asarray(ids)
    w = np.asarray(weights, dtype=np.float32)
    T, k = ids.shape
    d = x32.shape[1]
    per_slot = np.zeros((T, k, d), dtype=np.float32)
    for e in np.unique(ids[ids >= 0]):
        t_idx, j_idx = np.nonzero(ids == e)
        gate, up, down = experts[int(e)]
        y = swiglu_expert(x32[t_idx], gate, up, down, w[t_idx, j_idx], weight_before_down)
        per_slot[t_idx, j_idx] = y
    if out_per_slot:
        return per_slot
    acc = np.zeros((T, d), dtype=np.float64)
    for j in range(k):
        live = ids[:, j] >= 0
        scale = np.ones(T, dtype=np.float64) if weight_before_down else w[:, j].astype(np.float64)
        acc[live] += scale[live, None] * per_slot[live, j].astype(np.float64)
    return acc.astype(np.float32)


def rel_l2(ref: np.ndarray, got: np.ndarray) -> float:
    ref = np.asarray(ref, dtype=np.float64)
    got = np.asarray(got, dtype=np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(ref - got) / den) if den > 0 else float(np.linalg.norm(got))


# --- adaptive top-k router (loader/adaptive_topk.py) -------------------------

def _f32_sum(values: np.ndarray) -> np.float32:
    """np.sum of a short float32 vector, written out: numpy's pairwise sum
    (sequential from 0 below 8 elements; else eight strided accumulators
    combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the tail)."""
    a = np.asarray(values, np.float32)
    n = a.size
    if n < 8:
        r = np.float32(0.0)
        for v in a:
            r = np.float32(r + v)
        return r
    acc = [np.float32(v) for v in a[:8]]
    i = 8
    while i < n - n % 8:
        for j in range(8):
            acc[j] = np.float32(acc[j] + a[i + j])
        i += 8
    r = np.float32(np.float32(np.float32(acc[0] + acc[1]) + np.float32(acc[2] + acc[3])) +
                   np.float32(np.float32(acc[4] + acc[5]) + np.float32(acc[6] + acc[7])))
    while i < n:
        r = np.float32(r + a[i])
        i += 1
    return r


def adaptive_keep(sorted_scores: np.ndarray, threshold: float = 0.95) -> Tuple[int, np.float32]:
    """How many of the descending top-k scores to keep, and their float32 sum.

    Restates adaptive_topk_inclusive (loader/adaptive_topk.py:29-56) with the
    arithmetic numpy 2 gives it: total = float(np.sum(f32 scores)) (:47),
    target = threshold * total in float64 (:51), then the running sum and the
    comparison in float32 (a Python float meeting a float32 scalar is cast to
    float32, :53-56)."""
    s = np.asarray(sorted_scores, np.float32)
    if s.size == 0:
        return 0, np.float32(0.0)
    if not 0.0 < threshold <= 1.0:
        raise ValueError(f"threshold must be in (0, 1], got {threshold}")
    total = float(_f32_sum(s))
    if total <= 0:
        return 0, np.float32(0.0)
    target = np.float32(threshold * total)
    cum = np.float32(0.0)
    for i, v in enumerate(s):
        if np.float32(cum + v) > target:
            return i, cum
        cum = np.float32(cum + v)
    return int(s.size), cum


def router_topk(scores: np.ndarray, top_k: int, threshold: float = 0.95, renormalize: bool = True):
    """Router scores [T, E] -> (ids [T, k] int32, weights [T, k] float32, n_kept [T] int32).

    Top-k selection in descending score order as adaptive_topk_batch
    (loader/adaptive_topk.py:59-90; ties: lower expert id first, where the
    reference's unstable argsort leaves the order open), then adaptive_keep
    per token.  Dropped slots get id -1 and weight 0 (the op skips id < 0).
    Kept weights are the scores divided by their float32 sum when
    ``renormalize``, else the scores themselves."""
    scores = np.asarray(scores, np.float32)
    if scores.ndim != 2:
        raise ValueError(f"scores must be 2D, got {scores.ndim}D")
    T, E = scores.shape
    if top_k > E:
        raise ValueError(f"top_k={top_k} > n_experts={E}")
    order = np.argsort(-scores, axis=1, kind="stable")[:, :top_k]
    top = np.take_along_axis(scores, order, axis=1)
    ids = np.full((T, top_k), -1, np.int32)
    w = np.zeros((T, top_k), np.float32)
    n_kept = np.zeros(T, np.int32)
    for t in range(T):
        n, cum = adaptive_keep(top[t], threshold)
        n_kept[t] = n
        ids[t, :n] = order[t, :n]
        w[t, :n] = top[t, :n] / cum if renormalize else top[t, :n]
    return ids, w, n_kept
