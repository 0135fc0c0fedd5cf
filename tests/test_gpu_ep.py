"""Expert parallelism on two GPUs: NCCL all-to-all dispatch and return around
the local fused FFN, against the single-GPU fused op over all experts.

Each rank owns half of config 0's experts and routes its own batch (uneven
sizes, a skipped slot, one rank sending only to the other rank's experts).
The local FFN sees one row per routed slot, so its split-K partial sums group
differently from the single-GPU call: the bound is fp32 rounding (1e-5).
Skipped on a box with fewer than two GPUs."""

import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu
TOL = 1e-5


def _worker(rank, world, port, outdir, wbd, max_tokens):
    sys.path.insert(0, str(ROOT))
    import datetime
    import torch.distributed as dist
    from latent_b200 import ExpertFFN, ExpertSet, synth
    from latent_b200.ep import CudaEPOps, ExpertParallelFFN
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    cfg = synth.CONFIGS[0]
    E = cfg.n_expert
    e_local = E // world
    facs = synth.make_expert_factors(cfg, dev)
    full = ExpertSet(facs, device=dev, rank=cfg.rank)
    local = ExpertSet(facs[rank * e_local:(rank + 1) * e_local], device=dev, rank=cfg.rank)
    x, ids, w = synth.make_batch(cfg, dev, n_tokens=40 + 24 * rank, seed_offset=rank)
    ids[0, 1] = -1
    if rank == 1:
        ids = torch.where(ids >= 0, ids % e_local, ids)   # rank 1 sends only to rank 0
    ep = ExpertParallelFFN(E, CudaEPOps(local, E), max_tokens=max_tokens)
    errs = []
    for _ in range(2):                                   # the second call reuses the workspaces
        out = ep(x, ids, w, weight_before_down=wbd)
        ref = ExpertFFN(full, path="decode")(x, ids, w, weight_before_down=wbd)
        errs.append(float(torch.linalg.vector_norm((out - ref).double()) /
                          torch.linalg.vector_norm(ref.double())))
    np.save(Path(outdir) / f"r{rank}.npy", np.array(errs + [float(sum(ep.last_counts[1]))]))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.timeout(600)
@pytest.mark.parametrize("max_tokens", [None, 64], ids=["exact", "fixed-capacity"])
@pytest.mark.parametrize("wbd", [False, True])
def test_ep_two_gpus_match_single_gpu(cuda, wbd, max_tokens):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_worker, args=(world, _free_port(), tmp, wbd, max_tokens), nprocs=world, join=True,
                           start_method="spawn")
        res = [np.load(Path(tmp) / f"r{r}.npy") for r in range(world)]
    for rank, r in enumerate(res):
        assert max(r[:-1]) <= TOL, (rank, r)
    assert res[0][-1] > 0 and res[1][-1] >= 0
