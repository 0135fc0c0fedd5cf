"""Fixed-capacity expert-parallel blocks on one GPU: latent_ep_pack_fixed and
latent_ep_combine_fixed against the exact-split dispatch outputs they
re-place (no collective involved: the blocks are checked as laid out for 4
ranks)."""

import numpy as np
import pytest
import torch

from latent_b200 import ExpertSet, synth
from latent_b200.ep import CudaEPOps

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wbd", [False, True])
def test_pack_and_combine_fixed_match_exact_splits(cuda, wbd):
    dev = torch.device("cuda", 0)
    cfg = synth.CONFIGS[0]
    E, world = cfg.n_expert, 4
    el = E // world
    es = ExpertSet(synth.make_expert_factors(cfg, dev, experts=range(el)), device=dev, rank=cfg.rank)
    x, ids, w = synth.make_batch(cfg, dev, n_tokens=40)
    ids[0, 1] = -1
    ids[3] = torch.where(ids[3] >= 0, ids[3] % el, ids[3])
    T, k = ids.shape
    cap = T * min(k, el)
    ops = CudaEPOps(es, E)
    p = ops.dispatch(x, ids, w, wbd)
    rows, meta = ops.pack_fixed(p, world, cap)
    counts = p.expert_counts.view(world, el).sum(dim=1).cpu().numpy()
    off = np.concatenate([[0], np.cumsum(counts)])
    sx, se, sw = p.send_x.cpu(), p.send_expert.cpu().numpy(), p.send_weight.cpu().numpy()
    rows_c, meta_c = rows.cpu(), meta.cpu().numpy()
    for g in range(world):
        n = int(counts[g])
        assert n <= cap
        assert torch.equal(rows_c[g * cap:g * cap + n], sx[off[g]:off[g] + n])
        assert np.array_equal(meta_c[g * cap:g * cap + n, 0], se[off[g]:off[g] + n])
        assert np.array_equal(meta_c[g * cap:g * cap + n, 1], sw[off[g]:off[g] + n].view(np.int32))
        assert (meta_c[g * cap + n:(g + 1) * cap, 0] == -1).all()
    # returned blocks: random rows at the same placement; the exact-split combine reads them in send order
    y_rows = torch.randn((world * cap, cfg.n_embd), device=dev)
    idx = np.concatenate([g * cap + np.arange(int(counts[g])) for g in range(world)]).astype(np.int64)
    y_back = torch.zeros((max(T * k, 1), cfg.n_embd), device=dev)
    y_back[:idx.size] = y_rows[torch.from_numpy(idx).to(dev)]
    want = ops.combine(p, y_back)
    got = ops.combine_fixed(p, y_rows, world, cap)
    assert torch.equal(got, want)


def test_pack_fixed_overflow_keeps_the_first_rows_and_is_reported(cuda):
    """A token that routes one expert twice can overflow its block (cap
    assumes distinct experts per token): the block keeps its first cap rows
    in routed order, the rest are left out of the combine, and
    latent_ep_check reports LATENT_ERR_CAPACITY.  The next clean dispatch
    clears it."""
    from latent_b200 import _lib
    dev = torch.device("cuda", 0)
    cfg = synth.CONFIGS[0]
    E, world, T, k = cfg.n_expert, 8, 6, 2
    es = ExpertSet(synth.make_expert_factors(cfg, dev, experts=[0]), device=dev, rank=cfg.rank)
    x, _, _ = synth.make_batch(cfg, dev, n_tokens=T)
    ids = torch.zeros((T, k), dtype=torch.int32, device=dev)      # 2T rows to rank 0
    w = torch.full((T, k), 0.5, device=dev)
    cap = T * min(k, E // world)                                    # = T
    ops = CudaEPOps(es, E)
    p = ops.dispatch(x, ids, w, False)
    rows, meta = ops.pack_fixed(p, world, cap)
    with pytest.raises(_lib.LatentError) as info:
        ops.check(p)
    assert info.value.status == 10                                  # LATENT_ERR_CAPACITY
    assert torch.equal(rows[:cap].cpu(), p.send_x[:cap].cpu())
    assert (meta[:cap, 0] == 0).all() and (meta[cap:, 0] == -1).all()
    y_rows = torch.randn((world * cap, cfg.n_embd), device=dev)
    got = ops.combine_fixed(p, y_rows, world, cap)
    # the exact-split combine over send order, with the rows past cap zero
    y_back = torch.zeros((T * k, cfg.n_embd), device=dev)
    y_back[:cap] = y_rows[:cap]
    assert torch.equal(got, ops.combine(p, y_back))
    ok = ops.dispatch(x, torch.stack([ids[:, 0], ids[:, 0] + 1], dim=1).contiguous(), w, False)
    ops.pack_fixed(ok, world, cap)
    ops.check(ok)


@pytest.mark.parametrize("wbd", [False, True])
def test_merged_blocks_carry_the_same_rows_and_metadata(cuda, wbd):
    """latent_ep_pack_fixed_merged + latent_ep_unpack_fixed (rows and metadata in
    one buffer, one all-to-all) against the separate blocks of
    latent_ep_pack_fixed, with the exchange done by hand for 4 ranks: the
    receiving rank r gets block r of every sender (here one sender)."""
    dev = torch.device("cuda", 0)
    cfg = synth.CONFIGS[0]
    E, world = cfg.n_expert, 4
    el = E // world
    es = ExpertSet(synth.make_expert_factors(cfg, dev, experts=range(el)), device=dev, rank=cfg.rank)
    x, ids, w = synth.make_batch(cfg, dev, n_tokens=40)
    ids[0, 1] = -1
    T, k = ids.shape
    cap = T * min(k, el)
    ops = CudaEPOps(es, E)
    p = ops.dispatch(x, ids, w, wbd)
    rows, meta = ops.pack_fixed(p, world, cap)
    buf = ops.pack_fixed_merged(p, world, cap)
    assert buf.shape[0] == world
    for r in range(world):           # rank r receives block r of this sender: as if world senders sent alike
        recv = buf[r:r + 1].expand(world, -1).contiguous()
        rx, lids, rw = ops.unpack_fixed(recv, world, cap, x.dtype, r * el, wbd)
        blk_meta = meta[r * cap:(r + 1) * cap]
        live = blk_meta[:, 0] >= 0
        for g in range(world):
            sl = slice(g * cap, (g + 1) * cap)
            assert torch.equal(lids[sl, 0], torch.where(live, blk_meta[:, 0] - r * el, -1)), (r, g)
            assert torch.equal(rx[sl][live], rows[r * cap:(r + 1) * cap][live]), (r, g)
            want_w = blk_meta[:, 1].view(torch.float32) if wbd else torch.ones(cap, device=dev)
            assert torch.equal(rw[sl, 0][live], want_w[live]), (r, g)
