"""B200 runtime with the API of LATENT's CPU runtime (loader/latent_runtime.py:13-73).

Same names and argument meaning as the reference -- ``FactorPair``,
``load_pair``, ``project``, ``silu``, ``swiglu_expert``,
``dense_swiglu_expert`` -- plus the batched routed op ``moe_expert_ffn``
(GGML_OP_LATENT_EXPERT_FFN semantics).  Inputs may be numpy arrays (results
come back as numpy, like the reference) or torch tensors (results stay on
the device).  Factors stay packed on the device; nothing is dequantized to a
dense fp32 matrix on the fused path.  Every compute call goes through the
CUDA library; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Dict, Mapping, Optional, Tuple

import numpy as np
import torch

from . import _lib
from .format import ExpertSet, GroupedFactor, from_npz

__all__ = ["FactorPair", "load_pair", "project", "silu", "swiglu_expert", "dense_swiglu_expert",
           "moe_expert_ffn", "ExpertFFN", "workspace_bytes", "dequantize", "router_topk"]

_X_TYPES = {torch.float32: _lib.TYPE_F32, torch.float16: _lib.TYPE_F16, torch.bfloat16: _lib.TYPE_BF16}
_W_TYPES = {torch.float32: _lib.TYPE_F32, torch.float16: _lib.TYPE_F16}


def _device(device=None) -> torch.device:
    if device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("latent_b200 needs a CUDA device (no CPU fallback)")
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device(device)


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@dataclass
class FactorPair:
    """A low-rank pair W ~= A @ B kept packed on the device (reference FactorPair, latent_runtime.py:13-16).

    ``dense``: the matrix's dense-fallback copy (fp16 on the device) when it
    was loaded with ``load_pair(..., dense_fallback=True)``; ``project`` then
    uses it instead of the factors.
    """

    a: GroupedFactor
    b: GroupedFactor
    _sets: Dict[Tuple[int, int], ExpertSet] = field(default_factory=dict, repr=False, compare=False)
    dense: Optional[torch.Tensor] = None


def load_pair(arrays: Mapping[str, np.ndarray], name: str, device=None, dense_fallback: bool = False) -> FactorPair:
    """Reference-NPZ factors ``<name>.{a,b}.*`` -> device pair (latent_runtime.py:19-32).

    NF4 (group 32) is used when present, else INT8 (group 64); a missing
    factor raises ``KeyError`` like the reference.  With ``dense_fallback``
    the pair also carries ``<name>.dense_fallback`` when the artifact has one
    (loader/latent_loader.py:262-265; the reference runtime ignores it, as
    this function does by default).
    """
    dev = _device(device)
    pair = FactorPair(from_npz(arrays, name, "a").to(dev), from_npz(arrays, name, "b").to(dev))
    key = f"{name}.dense_fallback"
    if dense_fallback and key in arrays:
        pair.dense = torch.as_tensor(np.asarray(arrays[key])).to(device=dev, dtype=torch.float16).contiguous()
    return pair


def _matmul(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x [M, K] (f32/f16/bf16) @ w [K, N] (f32/f16) -> fp32 [M, N] by latent_dense_matmul."""
    if w.dtype not in _W_TYPES:
        w = w.float()
    if x.dtype not in _X_TYPES:
        x = x.float()
    M, K = x.shape
    if w.shape[0] != K:
        raise ValueError(f"matmul shapes {tuple(x.shape)} @ {tuple(w.shape)} do not match")
    N = w.shape[1]
    if K % 2:  # the kernel reads column pairs: a zero row/column pair changes no sum
        x = torch.nn.functional.pad(x, (0, 1))
        w = torch.nn.functional.pad(w, (0, 0, 0, 1))
    if N % 2:
        w = torch.nn.functional.pad(w, (0, 1))
    x, w = x.contiguous(), w.contiguous()
    Kp, Np = w.shape
    y = torch.empty((M, Np), dtype=torch.float32, device=w.device)
    _lib.check(_lib.lib().latent_dense_matmul(x.data_ptr(), _X_TYPES[x.dtype], w.data_ptr(), _W_TYPES[w.dtype],
                                              y.data_ptr(), M, Kp, Np, _stream_ptr(w.device)), "latent_dense_matmul")
    return y[:, :N] if Np != N else y


def _rows(x: torch.Tensor, k: int) -> Tuple[torch.Tensor, tuple]:
    lead = tuple(x.shape[:-1])
    return x.reshape(-1, k), lead


def dequantize(factor, expert: int = 0) -> torch.Tensor:
    """Dequantize one factor (GroupedFactor or StackedFactor expert) to fp32 on the device, bit-exact."""
    from .format import StackedFactor
    sf = factor if isinstance(factor, StackedFactor) else StackedFactor([factor], factor.lo.device)
    dev = sf.codes.device
    out = torch.empty((sf.rows, sf.cols), dtype=torch.float32, device=dev)
    qm = sf.qmatrix()
    _lib.check(_lib.lib().latent_dequantize(C.byref(qm), int(expert), out.data_ptr(), _stream_ptr(dev)),
               "latent_dequantize")
    return out


def pack_tiles(codes: torch.Tensor, scales: torch.Tensor, rows: int, cols: int):
    """Device repack of row-major stacked factor tensors into the tile-major layout.

    ``codes`` uint8 [E, rows, cols/2] and ``scales`` int16 (fp16 bits)
    [E, rows, cols/32] on a CUDA device, as the reference GGUF writer stores
    them (loader/write_latent_gguf.py:101-123); returns new (codes [E, g, 16],
    scales [E, g]) tensors in the order include/latent_ffn.h describes
    (latent_pack_tiles).
    """
    E = codes.shape[0]
    codes = codes.contiguous()
    scales = scales.contiguous()
    if codes.numel() != E * rows * cols // 2 or scales.numel() != E * rows * cols // 32:
        raise ValueError("codes/scales do not match [E, rows, cols]")
    g = rows * cols // 32
    dc = torch.empty((E, g, 16), dtype=torch.uint8, device=codes.device)
    ds = torch.empty((E, g), dtype=torch.int16, device=codes.device)
    _lib.check(_lib.lib().latent_pack_tiles(codes.data_ptr(), scales.data_ptr(), E, rows, cols, dc.data_ptr(),
                                            ds.data_ptr(), _stream_ptr(codes.device)), "latent_pack_tiles")
    return dc, ds


def _as_device_f32(x, dev) -> Tuple[torch.Tensor, bool]:
    if isinstance(x, np.ndarray) or not torch.is_tensor(x):
        return torch.as_tensor(np.asarray(x, dtype=np.float32)).to(dev), True
    return x.to(device=dev, dtype=torch.float32), False


def silu(x):
    """SiLU elementwise in fp32 on the device (latent_runtime.py:39-45)."""
    dev = _device(x.device if torch.is_tensor(x) and x.is_cuda else None)
    xt, host = _as_device_f32(x, dev)
    xt = xt.contiguous()
    y = torch.empty_like(xt)
    _lib.check(_lib.lib().latent_silu(xt.data_ptr(), y.data_ptr(), xt.numel(), _stream_ptr(dev)), "latent_silu")
    return y.cpu().numpy() if host else y


def project(x, pair: FactorPair):
    """(x @ A) @ B in fp32 (latent_runtime.py:35-36).

    A utility: A and B are dequantized bit-exactly by the CUDA library and
    multiplied by its fp32 CUDA-core GEMM (latent_dense_matmul); a pair
    loaded with its dense-fallback copy multiplies by that instead.  The
    fused expert path never materialises the factors.
    """
    dev = pair.a.lo.device
    xt, host = _as_device_f32(x, dev)
    x2, lead = _rows(xt, xt.shape[-1])
    if pair.dense is not None:
        y = _matmul(x2, pair.dense)
    else:
        y = _matmul(_matmul(x2, dequantize(pair.a)), dequantize(pair.b))
    y = y.reshape(*lead, y.shape[-1])
    return y.cpu().numpy() if host else y


def dense_swiglu_expert(x, gate, up, down, weight: float = 1.0, weight_before_down: bool = False):
    """Dense SwiGLU reference on the device (latent_runtime.py:62-73); the dense-fallback expert form."""
    dev = _device(gate.device if torch.is_tensor(gate) and gate.is_cuda else None)
    xt, host = _as_device_f32(x, dev)
    g, u, dn = (m.to(dev) if torch.is_tensor(m) and m.dtype in _W_TYPES else _as_device_f32(m, dev)[0]
                for m in (gate, up, down))
    x2, lead = _rows(xt, xt.shape[-1])
    h = silu(_matmul(x2, g)) * _matmul(x2, u)
    if weight_before_down:
        h = h * torch.as_tensor(weight, dtype=torch.float32, device=dev)
    y = _matmul(h, dn).reshape(*lead, dn.shape[-1])
    return y.cpu().numpy() if host else y


def _make_desc(experts: ExpertSet, T: int, k: int, x_type: int, w_type: int, flags: int, path: int) -> _lib.FfnDesc:
    d = _lib.FfnDesc()
    d.n_expert, d.n_embd, d.n_ff, d.rank = experts.n_expert, experts.n_embd, experts.n_ff, experts.rank
    d.n_tokens, d.top_k = T, k
    d.x_type, d.w_type, d.flags, d.path = x_type, w_type, flags, path
    for kind in ("gate_a", "gate_b", "up_a", "up_b", "down_a", "down_b"):
        setattr(d, kind, experts[kind].qmatrix())
    return d


_PATHS = {None: _lib.PATH_AUTO, "auto": _lib.PATH_AUTO, "decode": _lib.PATH_DECODE, "prefill": _lib.PATH_PREFILL}


def workspace_bytes(experts: ExpertSet, n_tokens: int, top_k: int, weight_before_down: bool = False,
                    out_per_slot: bool = False, path: Optional[str] = None,
                    x_dtype=torch.bfloat16, w_dtype=torch.float32) -> int:
    """Workspace the fused op needs for a batch of this shape (latent_expert_ffn_workspace_size)."""
    flags = (_lib.FLAG_WEIGHT_BEFORE_DOWN if weight_before_down else 0) | (_lib.FLAG_OUT_PER_SLOT if out_per_slot else 0)
    d = _make_desc(experts, n_tokens, top_k, _X_TYPES[x_dtype], _W_TYPES[w_dtype], flags, _PATHS[path])
    n = C.c_size_t(0)
    _lib.check(_lib.lib().latent_expert_ffn_workspace_size(C.byref(d), C.byref(n)), "workspace_size")
    return int(n.value)


class ExpertFFN:
    """The routed latent expert FFN over one ExpertSet (GGML_OP_LATENT_EXPERT_FFN).

    Calling it runs routing, the fused expert chain and the top-k combine on
    the current CUDA stream.  The workspace is allocated once per shape by
    this (host-side) object through torch and reused; the CUDA library
    itself allocates nothing.
    """

    def __init__(self, experts: ExpertSet, path: Optional[str] = None):
        self.experts = experts
        self.path = _PATHS[path]
        self._ws: Optional[torch.Tensor] = None
        self._last_desc: Optional[_lib.FfnDesc] = None
        self._dense = None      # dense-fallback tables (built on first use)
        self._dws: Optional[torch.Tensor] = None
        self._keep = None

    def _workspace(self, nbytes: int) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.experts.device)
        return self._ws

    def describe(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, out: torch.Tensor,
                 weight_before_down: bool = False, out_per_slot: bool = False) -> _lib.FfnDesc:
        """Validated descriptor for these device tensors (with workspace bound)."""
        ex = self.experts
        if x.dim() != 2 or x.shape[1] != ex.n_embd:
            raise ValueError(f"x must be [T, {ex.n_embd}], got {tuple(x.shape)}")
        T = x.shape[0]
        if ids.dim() != 2 or ids.shape[0] != T or ids.dtype != torch.int32:
            raise ValueError("ids must be int32 [T, k]")
        k = ids.shape[1]
        if weights.shape != ids.shape or weights.dtype not in _W_TYPES:
            raise ValueError("weights must be float32/float16 [T, k]")
        if x.dtype not in _X_TYPES:
            raise ValueError(f"x dtype {x.dtype} unsupported")
        for t in (x, ids, weights, out):
            if t.device != ex.device or not t.is_contiguous():
                raise ValueError("x, ids, weights and out must be contiguous tensors on the experts' device")
        flags = (_lib.FLAG_WEIGHT_BEFORE_DOWN if weight_before_down else 0) | \
                (_lib.FLAG_OUT_PER_SLOT if out_per_slot else 0)
        d = _make_desc(ex, T, k, _X_TYPES[x.dtype], _W_TYPES[weights.dtype], flags, self.path)
        n = C.c_size_t(0)
        _lib.check(_lib.lib().latent_expert_ffn_workspace_size(C.byref(d), C.byref(n)), "workspace_size")
        ws = self._workspace(int(n.value))
        d.x, d.ids, d.weights, d.out = x.data_ptr(), ids.data_ptr(), weights.data_ptr(), out.data_ptr()
        d.workspace, d.workspace_bytes = ws.data_ptr(), ws.numel()
        return d

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, weight_before_down: bool = False,
                 out_per_slot: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        T, k = ids.shape
        shape = (T, k, self.experts.n_embd) if out_per_slot else (T, self.experts.n_embd)
        if out is None:
            out = torch.empty(shape, dtype=torch.float32, device=self.experts.device)
        elif tuple(out.shape) != shape or out.dtype != torch.float32:
            raise ValueError(f"out must be float32 {shape}")
        if self.experts.dense:
            return self._call_mixed(x, ids, weights, weight_before_down, out_per_slot, out)
        d = self.describe(x, ids, weights, out, weight_before_down, out_per_slot)
        self._last_desc = d
        _lib.check(_lib.lib().latent_expert_ffn_forward(C.byref(d), _stream_ptr(self.experts.device)),
                   "latent_expert_ffn_forward")
        return out

    def _dense_tables(self):
        """latent_dense_expert entries of the set's dense-fallback experts (built once)."""
        if self._dense is None:
            es = self.experts
            flagged = sorted(es.dense)
            arr = (_lib.DenseExpert * len(flagged))()
            keep = []
            index = torch.full((es.n_expert,), -1, dtype=torch.int32)
            for i, e in enumerate(flagged):
                index[e] = i
                arr[i].expert, arr[i].rank = e, es.rank
                for m, name in enumerate(("gate", "up", "down")):
                    w = es.dense[e].get(name)
                    if w is not None:
                        arr[i].dense[m] = w.data_ptr()
                    else:  # the kind keeps its factors: exact fp32 A and B
                        a, b = dequantize(es[f"{name}_a"], e), dequantize(es[f"{name}_b"], e)
                        keep += [a, b]
                        arr[i].a[m], arr[i].b[m] = a.data_ptr(), b.data_ptr()
            self._dense = (arr, index.to(es.device), keep)
        return self._dense

    def _call_mixed(self, x, ids, weights, wbd, per_slot, out):
        """Latent experts through the fused op, dense-fallback experts through the dense kernels."""
        arr, index, _ = self._dense_tables()
        es = self.experts
        T, k = ids.shape
        dd = _lib.DenseDesc()
        dd.n_expert, dd.n_embd, dd.n_ff, dd.n_tokens, dd.top_k = es.n_expert, es.n_embd, es.n_ff, T, k
        dd.x_type, dd.w_type, dd.dense_type = _X_TYPES[x.dtype], _W_TYPES[weights.dtype], _lib.TYPE_F16
        dd.flags = (_lib.FLAG_WEIGHT_BEFORE_DOWN if wbd else 0) | (_lib.FLAG_OUT_PER_SLOT if per_slot else 0)
        dd.n_dense, dd.experts, dd.dense_index = len(arr), arr, index.data_ptr()
        dd.x, dd.ids, dd.weights, dd.out = x.data_ptr(), ids.data_ptr(), weights.data_ptr(), out.data_ptr()
        n = C.c_size_t(0)
        _lib.check(_lib.lib().latent_dense_workspace_size(C.byref(dd), C.byref(n)), "latent_dense_workspace_size")
        if self._dws is None or self._dws.numel() < n.value:
            self._dws = torch.empty(max(int(n.value), 256), dtype=torch.uint8, device=es.device)
        dd.workspace, dd.workspace_bytes = self._dws.data_ptr(), self._dws.numel()
        stream = _stream_ptr(es.device)
        ids_latent = torch.empty_like(ids)
        _lib.check(_lib.lib().latent_dense_experts_prepare(C.byref(dd), ids_latent.data_ptr(), stream),
                   "latent_dense_experts_prepare")
        d = self.describe(x, ids_latent, weights, out, wbd, per_slot)
        self._last_desc = d
        self._keep = ids_latent
        _lib.check(_lib.lib().latent_expert_ffn_forward(C.byref(d), stream), "latent_expert_ffn_forward")
        _lib.check(_lib.lib().latent_dense_experts_forward(C.byref(dd), stream), "latent_dense_experts_forward")
        return out

    def call_timed(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, events,
                   weight_before_down: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Like ``__call__``; records ``events`` (recorded torch.cuda.Event objects) around every kernel
        (layers without dense-fallback experts)."""
        if self.experts.dense:
            raise ValueError("call_timed serves layers without dense-fallback experts")
        T, k = ids.shape
        if out is None:
            out = torch.empty((T, self.experts.n_embd), dtype=torch.float32, device=self.experts.device)
        d = self.describe(x, ids, weights, out, weight_before_down, False)
        self._last_desc = d
        handles = (C.c_void_p * len(events))(*[ev.cuda_event for ev in events])
        _lib.check(_lib.lib().latent_expert_ffn_forward_timed(
            C.byref(d), _stream_ptr(self.experts.device), handles, len(events)), "latent_expert_ffn_forward_timed")
        return out

    def check(self) -> None:
        """Synchronises and raises if the last call recorded a device-side error
        (an expert id >= n_expert was routed, or a bounded wait ran out)."""
        if self._last_desc is not None:
            _lib.check(_lib.lib().latent_expert_ffn_check(C.byref(self._last_desc),
                                                          _stream_ptr(self.experts.device)), "device check")


def _to_dev(a, dev, dtype=None):
    if torch.is_tensor(a):
        return a.to(device=dev, dtype=dtype if dtype is not None else a.dtype).contiguous()
    arr = np.asarray(a)
    t = torch.from_numpy(np.ascontiguousarray(arr))
    return t.to(device=dev, dtype=dtype if dtype is not None else t.dtype).contiguous()


_OPS: Dict[int, ExpertFFN] = {}


def router_topk(scores: torch.Tensor, top_k: int, threshold: float = 0.95, renormalize: bool = True,
                logits: bool = False, expert_counts: bool = False):
    """Adaptive top-k routing on the device (latent_router_topk).

    scores: [T, E] fp32 router scores on a CUDA device.  Returns (ids [T, k]
    int32, weights [T, k] fp32, n_kept [T] int32): the top-k experts in
    descending score order, the tail beyond the reference's inclusive
    threshold rule dropped to id -1 / weight 0 (loader/adaptive_topk.py:29-90),
    kept weights renormalised to sum to 1 unless ``renormalize`` is False.
    The ids and weights feed ``ExpertFFN`` / ``moe_expert_ffn`` directly.
    With ``logits`` the scores are router logits and the softmax runs in the
    same kernel (latent_router_route); with ``expert_counts`` a fourth
    result holds the kept slots per expert [E] int32.
    Raises ValueError where the reference does (threshold outside (0, 1],
    top_k > n_experts, scores not 2-D)."""
    if not torch.is_tensor(scores) or scores.device.type != "cuda":
        raise ValueError("scores must be a CUDA tensor")
    if scores.dim() != 2:
        raise ValueError(f"scores must be 2D, got {scores.dim()}D")
    T, E = scores.shape
    if top_k > E:
        raise ValueError(f"top_k={top_k} > n_experts={E}")
    if top_k < 1:
        raise ValueError(f"top_k must be positive, got {top_k}")
    if not 0.0 < threshold <= 1.0:
        raise ValueError(f"threshold must be in (0, 1], got {threshold}")
    s = scores.to(torch.float32).contiguous()
    ids = torch.empty((T, top_k), dtype=torch.int32, device=s.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=s.device)
    n_kept = torch.empty(T, dtype=torch.int32, device=s.device)
    flags = (_lib.ROUTER_RENORMALIZE if renormalize else 0) | (_lib.ROUTER_SOFTMAX if logits else 0)
    counts = torch.empty(E, dtype=torch.int32, device=s.device) if expert_counts else None
    _lib.check(_lib.lib().latent_router_route(s.data_ptr(), T, E, top_k, float(threshold), flags, ids.data_ptr(),
                                              w.data_ptr(), n_kept.data_ptr(),
                                              counts.data_ptr() if counts is not None else None,
                                              _stream_ptr(s.device)), "latent_router_route")
    return (ids, w, n_kept, counts) if expert_counts else (ids, w, n_kept)


def moe_expert_ffn(x, ids, weights, experts: ExpertSet, weight_before_down: bool = False,
                   out_per_slot: bool = False, path: Optional[str] = None):
    """Batched routed expert FFN: out[t] = sum_j w[t,j] * swiglu_expert_{ids[t,j]}(x[t]).

    ``ids`` < 0 skip a slot.  numpy inputs give a numpy result.
    """
    host = not torch.is_tensor(x)
    dev = experts.device
    xt = _to_dev(x, dev, torch.float32 if host and np.asarray(x).dtype == np.float64 else None)
    it = _to_dev(ids, dev, torch.int32)
    wt = _to_dev(weights, dev, torch.float32 if (host or weights.dtype not in _W_TYPES) else None)
    key = id(experts) * 4 + _PATHS[path]
    op = _OPS.get(key)
    if op is None or op.experts is not experts:
        op = _OPS[key] = ExpertFFN(experts, path)
    y = op(xt, it, wt, weight_before_down, out_per_slot)
    return y.cpu().numpy() if host else y


def swiglu_expert(x, gate: FactorPair, up: FactorPair, down: FactorPair, weight=1.0,
                  weight_before_down: bool = False):
    """SwiGLU expert over packed factor pairs (latent_runtime.py:48-59).

    Returns silu((x@A_g)@B_g) * ((x@A_u)@B_u) [* weight] @ A_d @ B_d; the weight
    only enters when ``weight_before_down`` (the caller applies it otherwise).
    """
    key = (id(up), id(down))
    es = gate._sets.get(key)
    if es is None:
        es = gate._sets[key] = ExpertSet([{"gate_a": gate.a, "gate_b": gate.b, "up_a": up.a, "up_b": up.b,
                                           "down_a": down.a, "down_b": down.b}], device=gate.a.lo.device)
    host = not torch.is_tensor(x)
    xt = _to_dev(x, es.device, torch.float32 if host else None)
    one_d = xt.dim() == 1
    if one_d:
        xt = xt[None, :]
    T = xt.shape[0]
    ids = torch.zeros((T, 1), dtype=torch.int32, device=es.device)
    w = torch.as_tensor(weight, dtype=torch.float32, device=es.device) if weight_before_down else \
        torch.ones((), dtype=torch.float32, device=es.device)
    w = w.reshape(-1, 1).expand(T, 1).contiguous()
    y = moe_expert_ffn(xt, ids, w, es, weight_before_down=weight_before_down)
    if one_d:
        y = y[0]
    return y.cpu().numpy() if host else y
