"""Expert parallelism: the routed expert FFN sharded over ranks by expert.

Experts are contiguous per rank (rank g owns experts [g*E/G, (g+1)*E/G)).
One call, on every rank:
  1. dispatch (CUDA library): route the local batch by global expert id and
     pack one row per routed slot in expert order = destination-rank order;
  2. all-to-all of per-destination row counts, one host read of the counts
     (or, with a fixed token capacity, no count exchange: fixed-size blocks
     per destination whose unused rows carry expert id -1);
  3. all-to-all of the rows (x in its dtype) and of (expert id, weight);
  4. the fused latent FFN over the received rows with the local experts
     (top-1, weight 1 -- or the router weight before the down projection);
  5. all-to-all of the fp32 expert outputs back to the source ranks;
  6. combine (CUDA library): out[t] = sum_j w[t,j] * y_(t,j) in slot order.
Weights never move.  Every byte between GPUs goes through NCCL into local
HBM; no kernel reads peer memory.  The reference has no multi-GPU code.

The per-rank compute steps are behind a small ``ops`` interface so that the
collective bookkeeping can be exercised on CPU ranks (gloo) with a CPU test
double; the product ops are ``CudaEPOps``.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from .format import ExpertSet
from .runtime import ExpertFFN, _W_TYPES, _X_TYPES, _stream_ptr


@dataclass
class Packed:
    send_x: torch.Tensor        # [T*k, d] rows in expert order
    send_expert: torch.Tensor   # [T*k] int32 global expert id
    send_weight: torch.Tensor   # [T*k] float32
    expert_counts: torch.Tensor  # [E] int32
    state: object = None         # whatever combine needs
    overflow: bool = False       # a fixed-capacity block overflowed (host-side packing only)


class CudaEPOps:
    """Dispatch / local FFN / combine through the CUDA library."""

    def __init__(self, local_experts: ExpertSet, n_expert: int, path: Optional[str] = "decode"):
        self.local = local_experts
        self.n_expert = n_expert
        self.ffn = ExpertFFN(local_experts, path=path)
        self._ws: Optional[torch.Tensor] = None

    def _desc(self, x, ids, weights, wbd: bool) -> _lib.EpDesc:
        d = _lib.EpDesc()
        d.n_expert, d.n_embd = self.n_expert, x.shape[1]
        d.n_tokens, d.top_k = ids.shape
        d.x_type, d.w_type = _X_TYPES[x.dtype], _W_TYPES[weights.dtype]
        d.flags = _lib.FLAG_WEIGHT_BEFORE_DOWN if wbd else 0
        d.x, d.ids, d.weights = x.data_ptr(), ids.data_ptr(), weights.data_ptr()
        n = C.c_size_t()
        _lib.check(_lib.lib().latent_ep_workspace_size(C.byref(d), C.byref(n)), "latent_ep_workspace_size")
        if self._ws is None or self._ws.numel() < n.value:
            self._ws = torch.empty(max(int(n.value), 256), dtype=torch.uint8, device=x.device)
        d.workspace, d.workspace_bytes = self._ws.data_ptr(), self._ws.numel()
        return d

    def dispatch(self, x, ids, weights, wbd: bool) -> Packed:
        T, k = ids.shape
        dev = x.device
        p = Packed(torch.empty((max(T * k, 1), x.shape[1]), dtype=x.dtype, device=dev),
                   torch.empty(max(T * k, 1), dtype=torch.int32, device=dev),
                   torch.empty(max(T * k, 1), dtype=torch.float32, device=dev),
                   torch.empty(self.n_expert, dtype=torch.int32, device=dev))
        d = self._desc(x, ids, weights, wbd)
        d.send_x, d.send_expert, d.send_weight = p.send_x.data_ptr(), p.send_expert.data_ptr(), p.send_weight.data_ptr()
        d.expert_counts = p.expert_counts.data_ptr()
        _lib.check(_lib.lib().latent_ep_dispatch(C.byref(d), _stream_ptr(dev)), "latent_ep_dispatch")
        p.state = (x, ids, weights, wbd)
        return p

    def local_ffn(self, rx, local_ids, rw, wbd: bool) -> torch.Tensor:
        if rx.shape[0] == 0:
            return torch.empty((0, rx.shape[1]), dtype=torch.float32, device=rx.device)
        return self.ffn(rx, local_ids, rw, weight_before_down=wbd)

    def pack_fixed(self, p: Packed, world: int, cap: int):
        """Fixed-capacity send blocks: rows [world*cap, d] and meta [world*cap, 2] (id -1 marks unused rows)."""
        x, ids, weights, wbd = p.state
        rows = torch.empty((world * cap, x.shape[1]), dtype=x.dtype, device=x.device)
        meta = torch.empty((world * cap, 2), dtype=torch.int32, device=x.device)
        d = self._desc(x, ids, weights, wbd)
        d.send_x, d.send_expert, d.send_weight = p.send_x.data_ptr(), p.send_expert.data_ptr(), p.send_weight.data_ptr()
        _lib.check(_lib.lib().latent_ep_pack_fixed(C.byref(d), world, cap, rows.data_ptr(), meta.data_ptr(),
                                                   _stream_ptr(x.device)), "latent_ep_pack_fixed")
        return rows, meta

    def pack_fixed_merged(self, p: Packed, world: int, cap: int) -> torch.Tensor:
        """The fixed-capacity blocks with rows and (id, weight) metadata in one byte buffer [world, block]."""
        x, ids, weights, wbd = p.state
        d = self._desc(x, ids, weights, wbd)
        d.send_x, d.send_expert, d.send_weight = p.send_x.data_ptr(), p.send_expert.data_ptr(), p.send_weight.data_ptr()
        need = C.c_size_t()
        lib, stream = _lib.lib(), _stream_ptr(x.device)
        _lib.check(lib.latent_ep_pack_fixed_merged(C.byref(d), world, cap, None, 0, C.byref(need), stream), "size")
        buf = torch.empty((world, need.value // world), dtype=torch.uint8, device=x.device)
        _lib.check(lib.latent_ep_pack_fixed_merged(C.byref(d), world, cap, buf.data_ptr(), buf.numel(), None,
                                                   stream), "latent_ep_pack_fixed_merged")
        return buf

    def unpack_fixed(self, buf: torch.Tensor, world: int, cap: int, x_dtype, base: int, wbd: bool):
        """Received merged blocks -> (x rows [world*cap, d], local ids [world*cap, 1], weights [world*cap, 1])."""
        dev = buf.device
        d = self.local.n_embd
        x_out = torch.empty((world * cap, d), dtype=x_dtype, device=dev)
        ids = torch.empty((world * cap, 1), dtype=torch.int32, device=dev)
        w = torch.empty((world * cap, 1), dtype=torch.float32, device=dev)
        _lib.check(_lib.lib().latent_ep_unpack_fixed(
            buf.data_ptr(), world, cap, d, _X_TYPES[x_dtype], base, self.local.n_expert,
            _lib.FLAG_WEIGHT_BEFORE_DOWN if wbd else 0, x_out.data_ptr(), ids.data_ptr(), w.data_ptr(), None,
            _stream_ptr(dev)), "latent_ep_unpack_fixed")
        return x_out, ids, w

    def combine_fixed(self, p: Packed, y_rows: torch.Tensor, world: int, cap: int) -> torch.Tensor:
        x, ids, weights, wbd = p.state
        out = torch.empty((ids.shape[0], x.shape[1]), dtype=torch.float32, device=x.device)
        d = self._desc(x, ids, weights, wbd)
        _lib.check(_lib.lib().latent_ep_combine_fixed(C.byref(d), world, cap, y_rows.data_ptr(), out.data_ptr(),
                                                      _stream_ptr(x.device)), "latent_ep_combine_fixed")
        return out

    def check(self, p: Packed) -> None:
        """Synchronise and raise on device-side errors of this dispatch (an
        expert id out of range, a fixed-capacity block that overflowed)."""
        x, ids, weights, wbd = p.state
        d = self._desc(x, ids, weights, wbd)
        _lib.check(_lib.lib().latent_ep_check(C.byref(d), _stream_ptr(x.device)), "latent_ep_check")

    def combine(self, p: Packed, y_back: torch.Tensor) -> torch.Tensor:
        x, ids, weights, wbd = p.state
        out = torch.empty((ids.shape[0], x.shape[1]), dtype=torch.float32, device=x.device)
        d = self._desc(x, ids, weights, wbd)
        d.y_back, d.out = y_back.data_ptr(), out.data_ptr()
        _lib.check(_lib.lib().latent_ep_combine(C.byref(d), _stream_ptr(x.device)), "latent_ep_combine")
        return out


class ExpertParallelFFN:
    """Routed expert FFN with experts sharded over the ranks of ``group``.

    Two exchange modes:
      * ``max_tokens=None``: exact splits.  Per-destination row counts are
        exchanged first and read on the host to size the row all-to-alls.
      * ``max_tokens=M`` (M = the most tokens any rank passes in one call, the
        same on every rank): fixed-capacity splits, no host read.  Each rank
        sends every destination a block of ``cap = M * min(k, E/G)`` rows
        (a token routes at most that many slots to one rank); rows past a
        destination's count carry expert id -1, which the fused op skips.
        The whole call is stream-ordered, so consecutive calls pipeline and
        the call can be captured with its collectives.  A batch in which a
        token routes one expert twice can overflow a block: its extra rows
        are left out of the exchange and the combine, and ``check()`` (a
        host synchronisation) raises LATENT_ERR_CAPACITY.
    """

    def __init__(self, n_expert: int, ops, group=None, max_tokens: Optional[int] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_expert % self.world:
            raise ValueError(f"{n_expert} experts do not split evenly over {self.world} ranks")
        if max_tokens is not None and max_tokens < 1:
            raise ValueError(f"max_tokens must be positive, got {max_tokens}")
        # Every rank must size the fixed blocks alike, or the all-to-alls
        # disagree on their splits: compare once, here, on the host.
        seen = [None] * self.world
        dist.all_gather_object(seen, max_tokens, group=group)
        if any(m != max_tokens for m in seen):
            raise ValueError(f"max_tokens differs across ranks: {seen}")
        self.n_expert = n_expert
        self.e_local = n_expert // self.world
        self.base = self.rank * self.e_local
        self.ops = ops
        self.max_tokens = max_tokens
        self._counts = None
        self._pos = None
        self._last = None

    def check(self) -> None:
        """Synchronise and raise if the last call recorded a device-side error
        (an expert id out of range, or a fixed-capacity block overflow)."""
        if self._last is not None and hasattr(self.ops, "check"):
            self.ops.check(self._last)
        elif self._last is not None and getattr(self._last, "overflow", False):
            raise _lib.LatentError(10, "fixed-capacity exchange")

    @property
    def last_counts(self):
        """(rows sent to each rank, rows received from each rank) of the last call, as lists."""
        if self._counts is None:
            return None
        sc, rc = self._counts
        if torch.is_tensor(sc):
            both = torch.stack([sc.to(torch.int64), rc.to(torch.int64)]).cpu()
            sc, rc = both[0].tolist(), both[1].tolist()
            self._counts = (sc, rc)
        return sc, rc

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                 weight_before_down: bool = False) -> torch.Tensor:
        if self.max_tokens is not None:
            return self._call_fixed(x, ids, weights, weight_before_down)
        G, d = self.world, x.shape[1]
        p = self.ops.dispatch(x, ids, weights, weight_before_down)
        send_counts = p.expert_counts.view(G, self.e_local).sum(dim=1).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        both = torch.stack([send_counts, recv_counts]).cpu()
        sc, rc = both[0].tolist(), both[1].tolist()
        self._counts = (sc, rc)
        self._last = p
        n_send, n_recv = sum(sc), sum(rc)
        recv_x = torch.empty((n_recv, d), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(recv_x, p.send_x[:n_send].contiguous(), rc, sc, group=self.group)
        meta = torch.stack([p.send_expert[:n_send], p.send_weight[:n_send].view(torch.int32)], dim=1).contiguous()
        recv_meta = torch.empty((n_recv, 2), dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_meta, meta, rc, sc, group=self.group)
        local_ids = (recv_meta[:, 0] - self.base).to(torch.int32).reshape(-1, 1).contiguous()
        if weight_before_down:
            rw = recv_meta[:, 1].contiguous().view(torch.float32).reshape(-1, 1).contiguous()
        else:
            rw = torch.ones((n_recv, 1), dtype=torch.float32, device=x.device)
        y = self.ops.local_ffn(recv_x, local_ids, rw, weight_before_down)
        y_back = torch.empty((max(n_send, 1), d), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(y_back[:n_send], y.contiguous(), sc, rc, group=self.group)
        return self.ops.combine(p, y_back)

    def _call_fixed(self, x, ids, weights, wbd):
        G, d = self.world, x.shape[1]
        T, k = ids.shape
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens}")
        cap = self.max_tokens * min(k, self.e_local)
        dev = x.device
        p = self.ops.dispatch(x, ids, weights, wbd)
        send_counts = p.expert_counts.view(G, self.e_local).sum(dim=1).to(torch.int64)
        fused = hasattr(self.ops, "pack_fixed")
        if hasattr(self.ops, "pack_fixed_merged"):
            # rows and their (id, weight) metadata in one all-to-all
            send = self.ops.pack_fixed_merged(p, G, cap)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
            recv_x, local_ids, rw = self.ops.unpack_fixed(recv, G, cap, x.dtype, self.base, wbd)
            y = self.ops.local_ffn(recv_x, local_ids, rw, wbd)
            y_pad = torch.empty((G * cap, d), dtype=torch.float32, device=dev)
            dist.all_to_all_single(y_pad, y.contiguous(), group=self.group)
            self._counts = (send_counts, (local_ids.view(G, cap) >= 0).sum(dim=1))
            self._last = p
            return self.ops.combine_fixed(p, y_pad, G, cap)
        if fused:
            send_x, send_meta = self.ops.pack_fixed(p, G, cap)
        else:
            # the same placement from torch index kernels (ops without a fused pack, e.g. CPU test doubles)
            dst = self._fixed_rows(p, send_counts, G, cap)
            send_x = torch.empty((G * cap + 1, d), dtype=x.dtype, device=dev)
            send_x.index_copy_(0, dst, p.send_x)
            meta = torch.stack([p.send_expert[:dst.numel()], p.send_weight[:dst.numel()].view(torch.int32)], dim=1)
            send_meta = torch.full((G * cap + 1, 2), -1, dtype=torch.int32, device=dev)
            send_meta.index_copy_(0, dst, meta)
        recv_x = torch.empty((G * cap, d), dtype=x.dtype, device=dev)
        dist.all_to_all_single(recv_x, send_x[:G * cap], group=self.group)
        recv_meta = torch.empty((G * cap, 2), dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_meta, send_meta[:G * cap], group=self.group)
        rid = recv_meta[:, 0]
        local_ids = torch.where(rid >= 0, rid - self.base, rid).reshape(-1, 1).contiguous()
        if wbd:
            rw = recv_meta[:, 1].contiguous().view(torch.float32).reshape(-1, 1).contiguous()
        else:
            rw = torch.ones((G * cap, 1), dtype=torch.float32, device=dev)
        y = self.ops.local_ffn(recv_x, local_ids, rw, wbd)
        y_pad = torch.empty((G * cap, d), dtype=torch.float32, device=dev)
        dist.all_to_all_single(y_pad, y.contiguous(), group=self.group)
        self._counts = (send_counts, (rid.view(G, cap) >= 0).sum(dim=1))
        self._last = p
        if fused:
            return self.ops.combine_fixed(p, y_pad, G, cap)
        # rows that did not fit their block (dst = G*cap) read a zero row
        y_ext = torch.cat([y_pad, y_pad.new_zeros((1, d))])
        return self.ops.combine(p, y_ext.index_select(0, dst))

    def _fixed_rows(self, p, send_counts, G: int, cap: int) -> torch.Tensor:
        """Block row of every routed position (G*cap past the routed rows: a discard row)."""
        P = p.send_x.shape[0]
        dev = p.send_x.device
        if self._pos is None or self._pos.numel() < P or self._pos.device != dev:
            self._pos = torch.arange(max(P, 1), dtype=torch.int64, device=dev)
        pos = self._pos[:P]
        end = torch.cumsum(send_counts, 0)
        g = torch.searchsorted(end, pos, right=True)
        gc = g.clamp(max=G - 1)
        slot = pos - (end - send_counts)[gc]
        keep = (g < G) & (slot < cap)
        p.overflow = bool((send_counts > cap).any())
        return torch.where(keep, gc * cap + slot, torch.full_like(pos, G * cap))
