"""Small fixed workloads for profiling one kernel at a time.

    python -m latent_b200.profile_cases router    # k_router_topk, config 3 routing shape (16384 x 256, top-8)
    python -m latent_b200.profile_cases prefill   # the prefill chain on config 2 (k_pf_* kernels)

Each case builds its inputs, runs the op a few times on cuda:0 and exits;
point a profiler's kernel filter and launch skip at the launch of interest.
"""

from __future__ import annotations

import sys

import torch


def router(calls: int = 5) -> None:
    from latent_b200 import router_topk
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    scores = torch.softmax(torch.randn((16384, 256), generator=g, device=dev), dim=1)
    for _ in range(calls):
        ids, w, nk = router_topk(scores, 8)
    torch.cuda.synchronize()
    print(f"router: mean kept {float(nk.float().mean()):.3f} of 8")


def prefill(calls: int = 3) -> None:
    from latent_b200 import ExpertFFN, synth
    dev = torch.device("cuda", 0)
    cfg = synth.CONFIGS[2]
    es = synth.make_expert_set(cfg, device=dev)
    x, ids, w = synth.make_batch(cfg, dev)
    op = ExpertFFN(es, path="prefill")
    for _ in range(calls):
        y = op(x, ids, w)
    op.check()
    torch.cuda.synchronize()
    print(f"prefill: mean |y| {float(y.abs().mean()):.4e}")


if __name__ == "__main__":
    cases = {"router": router, "prefill": prefill}
    if len(sys.argv) != 2 or sys.argv[1] not in cases:
        raise SystemExit(f"usage: python -m latent_b200.profile_cases {{{'|'.join(cases)}}}")
    torch.cuda.set_device(0)
    cases[sys.argv[1]]()
