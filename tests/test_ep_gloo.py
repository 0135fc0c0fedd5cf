"""Expert-parallel dispatch/all-to-all/combine bookkeeping on CPU ranks (gloo).

The per-rank compute (pack, local experts, combine) is a CPU test double
built on the oracle, so that the collective logic of ExpertParallelFFN --
count exchange, uneven splits, row ordering, weight transport, the return
path -- is checked against the single-process oracle without a GPU.
"""

import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


class CpuEPOps:
    def __init__(self, table, n_expert, base):
        self.table, self.E, self.base = table, n_expert, base

    def dispatch(self, x, ids, w, wbd):
        import oracle as O
        from latent_b200.ep import Packed
        T, k = ids.shape
        counts, offsets, order = O.route(ids.numpy(), self.E)
        pos = np.full(T * k, -1, np.int64)
        pos[order] = np.arange(order.size)
        send_x = x[torch.from_numpy(order // k)] if order.size else torch.zeros((0, x.shape[1]), dtype=x.dtype)
        return Packed(send_x.contiguous(), torch.from_numpy(ids.numpy().ravel()[order].astype(np.int32)),
                      torch.from_numpy(w.numpy().ravel()[order].astype(np.float32)),
                      torch.from_numpy(counts.astype(np.int32)), (ids, w, pos, wbd))

    def local_ffn(self, rx, local_ids, rw, wbd):
        import oracle as O
        y = np.zeros((rx.shape[0], rx.shape[1]), np.float32)
        lids = local_ids.numpy()[:, 0]
        for e in np.unique(lids[lids >= 0]):
            rows = lids == e
            y[rows] = O.swiglu_expert(rx.numpy()[rows], *self.table[self.base + int(e)], rw.numpy()[rows, 0], wbd)
        return torch.from_numpy(y)

    def combine(self, p, y_back):
        ids, w, pos, wbd = p.state
        T, k = ids.shape
        out = np.zeros((T, y_back.shape[1]), np.float64)
        yb = y_back.numpy()
        for t in range(T):
            for j in range(k):
                q = pos[t * k + j]
                if q >= 0:
                    out[t] += (1.0 if wbd else float(w[t, j])) * yb[q].astype(np.float64)
        return torch.from_numpy(out.astype(np.float32))


def _table(E, d, f, r):
    rng = np.random.default_rng(7)
    mk = lambda m, n: (rng.standard_normal((m, n)) * 0.2).astype(np.float32)
    return [((mk(d, r), mk(r, f)), (mk(d, r), mk(r, f)), (mk(f, r), mk(r, d))) for _ in range(E)]


def _worker(rank, world, port, outdir, wbd, max_tokens):
    sys.path.insert(0, str(ROOT))
    import oracle as O
    from latent_b200.ep import ExpertParallelFFN
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    E, d, f, r, k = 4, 64, 96, 32, 2
    table = _table(E, d, f, r)
    rng = np.random.default_rng(100 + rank)
    T = 7 + 3 * rank                       # uneven batches
    x = rng.standard_normal((T, d)).astype(np.float32)
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    ids[0, 1] = -1                          # skipped slot
    if rank == 1:
        ids[:, :] = np.where(ids >= 0, ids % 2, ids)   # rank 1 routes only to rank 0's experts
    w = rng.random((T, k)).astype(np.float32)
    ops = CpuEPOps(table, E, base=rank * (E // world))
    ep = ExpertParallelFFN(E, ops, max_tokens=max_tokens)
    out = ep(torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(w), weight_before_down=wbd).numpy()
    ref = O.moe_forward(x, ids, w, table, weight_before_down=wbd)
    np.save(Path(outdir) / f"r{rank}.npy", np.array([O.rel_l2(ref, out), float(sum(ep.last_counts[1]))]))
    dist.barrier()
    dist.destroy_process_group()


def _over_capacity(rank, world, port, outdir):
    sys.path.insert(0, str(ROOT))
    from latent_b200.ep import ExpertParallelFFN
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = ExpertParallelFFN(4, None, max_tokens=4)
    try:
        ep(torch.zeros((5, 8)), torch.zeros((5, 2), dtype=torch.int32), torch.ones((5, 2)))
        msg = "no error"
    except ValueError as e:
        msg = str(e)
    (Path(outdir) / f"r{rank}.txt").write_text(msg)
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("max_tokens", [None, 10, 16], ids=["exact", "cap10", "cap16"])
@pytest.mark.parametrize("wbd", [False, True])
def test_ep_two_cpu_ranks_match_single_process_oracle(wbd, max_tokens):
    """Exact splits, and fixed-capacity blocks (10 = the larger batch; 16 leaves spare rows)."""
    world = 2
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_worker, args=(world, _free_port(), tmp, wbd, max_tokens), nprocs=world, join=True,
                           start_method="spawn")
        res = [np.load(Path(tmp) / f"r{r}.npy") for r in range(world)]
    for rank, (err, n_recv) in enumerate(res):
        assert err < 1e-6, (rank, err)
    assert res[1][1] >= 0 and res[0][1] > 0   # rank 0 received rows from both ranks


def test_ep_fixed_capacity_rejects_larger_batch():
    world = 2
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_over_capacity, args=(world, _free_port(), tmp), nprocs=world, join=True,
                           start_method="spawn")
        for r in range(world):
            assert "max_tokens" in (Path(tmp) / f"r{r}.txt").read_text()


# ---- failure paths: made on the host, never on a device -------------------

def _run_ranks(fn, world, tmp, deadline=90.0):
    """Start `world` spawned ranks running fn(rank, world, port, tmp);
    fail (after killing them) if they have not all ended within `deadline` s."""
    import time
    tmp = str(tmp)
    ctx = mp.start_processes(fn, args=(world, _free_port(), tmp), nprocs=world, join=False,
                             start_method="spawn")
    end = time.monotonic() + deadline
    try:
        while not ctx.join(timeout=1.0):
            if time.monotonic() > end:
                pytest.fail(f"ranks still running after {deadline} s")
    finally:
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
    return tmp


def _rank_leaves(rank, world, port, outdir):
    """Rank 1 leaves between steps (after the first call); rank 0 makes a
    second call, whose first collective must end in an error, not a hang."""
    import datetime
    sys.path.insert(0, str(ROOT))
    from latent_b200.ep import ExpertParallelFFN
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    E, d, f, r, k = 4, 64, 96, 32, 2
    ops = CpuEPOps(_table(E, d, f, r), E, base=rank * (E // world))
    ep = ExpertParallelFFN(E, ops)
    x = torch.randn((6, d))
    ids = torch.randint(0, E, (6, k), dtype=torch.int32)
    w = torch.rand((6, k))
    ep(x, ids, w)                                     # step 1: both ranks
    if rank == 1:
        (Path(outdir) / "r1.txt").write_text("left")
        os._exit(0)                                   # leaves without a word to the others
    try:
        ep(x, ids, w)                                 # step 2: rank 1 is gone
        msg = "no error"
    except Exception as e:                            # gloo: connection closed or timed out
        msg = "raised " + type(e).__name__
    (Path(outdir) / "r0.txt").write_text(msg)
    os._exit(0)


def test_ep_rank_that_leaves_ends_the_next_collective_with_an_error(tmp_path):
    tmp = _run_ranks(_rank_leaves, 2, tmp_path)
    assert (Path(tmp) / "r1.txt").read_text() == "left"
    assert (Path(tmp) / "r0.txt").read_text().startswith("raised")


def _mismatched_caps(rank, world, port, outdir):
    sys.path.insert(0, str(ROOT))
    from latent_b200.ep import ExpertParallelFFN
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ExpertParallelFFN(4, None, max_tokens=8 + 4 * rank)
        msg = "no error"
    except ValueError as e:
        msg = str(e)
    (Path(outdir) / f"r{rank}.txt").write_text(msg)
    dist.destroy_process_group()


def test_ep_fixed_capacity_mismatch_across_ranks_is_rejected_on_every_rank(tmp_path):
    tmp = _run_ranks(_mismatched_caps, 2, tmp_path)
    for r in range(2):
        assert "differs across ranks" in (Path(tmp) / f"r{r}.txt").read_text()


def _repeated_ids(rank, world, port, outdir):
    """Tokens that route one expert twice overflow the fixed blocks (cap =
    M * min(k, E/G) assumes distinct experts per token): with E=2 over 2
    ranks and k=2, cap = M, and T tokens that all route expert 0 twice send
    2T rows to rank 0.  The block keeps the first T rows in routed order (the
    first T/2 tokens, both slots); the rest are left out of the exchange and
    the combine, and check() reports the overflow."""
    sys.path.insert(0, str(ROOT))
    import oracle as O
    from latent_b200 import _lib
    from latent_b200.ep import ExpertParallelFFN
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    E, d, f, r, k, T = 2, 64, 96, 32, 2, 4
    table = _table(E, d, f, r)
    ep = ExpertParallelFFN(E, CpuEPOps(table, E, base=rank), max_tokens=T)
    x = torch.randn((T, d), generator=torch.Generator().manual_seed(rank))
    ids = torch.zeros((T, k), dtype=torch.int32)
    w = torch.full((T, k), 0.5)
    out = ep(x, ids, w).numpy()
    ref = O.moe_forward(x.numpy(), ids.numpy(), w.numpy(), table)
    kept = O.rel_l2(ref[:T // 2], out[:T // 2]) < 1e-6 and not out[T // 2:].any()
    try:
        ep.check()
        msg = "no error"
    except _lib.LatentError as e:
        msg = f"status {e.status}"
    (Path(outdir) / f"r{rank}.txt").write_text(f"{kept} {msg}")
    dist.destroy_process_group()


def test_ep_fixed_capacity_overflow_is_dropped_and_reported(tmp_path):
    tmp = _run_ranks(_repeated_ids, 2, tmp_path)
    for r in range(2):
        assert (Path(tmp) / f"r{r}.txt").read_text() == "True status 10"
