#!/usr/bin/env python3
"""Benchmark of the fused latent expert FFN (BASELINE metric: routed tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]
    python bench.py --only decode|prefill|router|sweep   # one leg alone (profiling runs)

A step is one pass of the hot path -- routing, then the fused kernel that runs
the four-phase latent SwiGLU chain over every routed (token, expert) pair and
the top-k combine -- over
one batch of the config's synthetic layer (``latent_b200.synth``, seeded).
Default workload: config 1 (DeepSeek-V2-Lite-shaped decode: 64 experts,
d=2048, f=1408, rank 256, top-6, 32 tokens, bf16 activations).

``value``: routed pairs (id >= 0) of all ranks / max-over-ranks mean device
time per step, inputs resident in HBM, L2 flushed (256 MiB write) before every
step outside the timed events (a write of one buffer, then a read of another,
so that no dirty flush lines are written back inside the timed region).  ``e2e``: the same metric through the public
op with pinned host buffers: H2D of x/ids/weights and D2H of the output are
inside the timed region.  ``roofline``: the dominant kernel's algorithmic
bytes / its mean duration (CUDA events recorded between the library's kernel
launches), against MEASURED_PEAKS.json; ``traffic`` is null (DRAM bytes are
not measured inside this run; profiles/ holds the ncu figures).
``cpu_baseline`` / ``--impl reference``: the reference CPU runtime's
algorithm (the numpy oracle port) on the host cores.  Both arms print the
same ``config`` dict; how the job is spread over GPUs is the top-level
``parallel`` key.  Extra legs of the default 1-GPU run: ``prefill`` (config
2, tensor-core path), ``router`` (config 3 routing shape) and ``sweep``
(config 4 decode shapes: ranks 64/256/512, batches 1..256).
"""

from __future__ import annotations

import os

_NCPU = os.cpu_count() or 1
for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
    os.environ.setdefault(_v, str(_NCPU))
# NCCL's own messages (e.g. its version line) go to stderr: stdout carries the one JSON line
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

import argparse
import datetime
import json
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "latent MoE-FFN routed tokens/s/GPU, decode & prefill; % HBM/tensor roofline"
UNIT = "routed tokens/s"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="bound on the CPU baseline's timed work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-2 prefill leg of the default run")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config-4 decode sweep of the default run")
    ap.add_argument("--only", choices=["decode", "prefill", "router", "sweep"],
                    help="run one leg alone on cuda:0 and print its JSON (no CPU baseline, no e2e); "
                         "for profiling one kernel at a time")
    ap.add_argument("--ep-exact", action="store_true",
                    help="expert parallel: exact splits with a host read of the counts (default: fixed capacity)")
    ap.add_argument("--ep-eager", action="store_true",
                    help="expert parallel: launch the fixed-capacity step eagerly instead of replaying it "
                         "as one captured CUDA graph (the default)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allreduce_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allreduce_sum(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


PHASES = ["route (k_route_single)", "fused expert chain (k_chain)"]
KINDS = ("gate_a", "up_a", "gate_b", "up_b", "down_a", "down_b")


class L2Flush:
    """Writes a 256 MiB buffer, then reads another one: L2 ends up holding clean, unrelated lines."""

    def __init__(self, dev):
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.sink = self.r.sum()


def workload(cfg_id: int, device, rank: int = 0):
    from latent_b200 import synth
    cfg = synth.CONFIGS[cfg_id]
    t0 = time.perf_counter()
    es = synth.make_expert_set(cfg, device=device)
    x, ids, w = synth.make_batch(cfg, device, seed_offset=rank)
    torch.cuda.synchronize()
    return cfg, es, x, ids, w, time.perf_counter() - t0


def kind_bytes(es, kinds, experts):
    return sum(es[k].nbytes(experts) + es[k].int8_bytes(experts) for k in kinds)


def config_json(cfg, ids):
    """The workload, identical in both arms (how it is spread over GPUs is reported beside it)."""
    routed = int((ids >= 0).sum())
    return {"workload": cfg.name, "n_expert": cfg.n_expert, "n_embd": cfg.n_embd, "n_ff": cfg.n_ff,
            "rank": cfg.rank, "top_k": cfg.top_k, "tokens_per_gpu": int(ids.shape[0]),
            "routed_per_gpu": routed, "x_dtype": str(cfg.x_dtype).replace("torch.", ""),
            "quant": "NF4 g32 + per-group INT8 below 20 dB",
            "l2": "flushed before every step (256 MiB write, then 256 MiB read of another buffer)",
            "seed": cfg.seed}


def cpu_leg(cfg, es, x, ids, w, seconds: float, min_steps: int = 3):
    """The reference runtime's algorithm (oracle port, numpy) on the host cores: steady-state forward
    over the batch with factors pre-dequantized (the dequant time is reported separately)."""
    import oracle as O
    touched = sorted(set(ids[ids >= 0].cpu().tolist()))
    t0 = time.perf_counter()
    table = [None] * cfg.n_expert
    for e in touched:
        pairs = []
        for n in ("gate", "up", "down"):
            fa, fb = es[f"{n}_a"].expert(e), es[f"{n}_b"].expert(e)
            pairs.append(tuple(O.decode_grouped(f.lo.numpy(), f.hi.numpy(), f.scales.numpy().view(np.uint16),
                                                f.is_int8.numpy(), f.rows, f.cols) for f in (fa, fb)))
        table[e] = tuple(pairs)
    dequant_s = time.perf_counter() - t0
    xs, ids_np, w_np = x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()
    O.moe_forward(xs, ids_np, w_np, table)      # warm-up
    times = []
    t_start = time.perf_counter()
    while len(times) < min_steps or (time.perf_counter() - t_start) < seconds:
        t1 = time.perf_counter()
        O.moe_forward(xs, ids_np, w_np, table)
        times.append(time.perf_counter() - t1)
        if len(times) >= 10000:
            break
    routed = int((ids >= 0).sum())
    step = statistics.mean(times)
    return {"value": routed / step, "unit": UNIT, "cores": _NCPU, "kind": "port",
            "sample": f"{len(times)} full batches of {ids.shape[0]} tokens ({routed} routed pairs), "
                      f"{len(touched)} experts pre-dequantized in {dequant_s:.2f} s",
            "ms_per_step": step * 1e3, "dequant_s": dequant_s}


def run_ours(args, world, rank, local):
    from latent_b200 import ExpertFFN
    dev = torch.device("cuda", local)
    cfg, es, x, ids, w, gen_s = workload(args.config, dev, rank)
    op = ExpertFFN(es, path="decode")
    R = int(ids.shape[0] * ids.shape[1])
    routed = int((ids >= 0).sum())
    touched = sorted(set(ids[ids >= 0].cpu().tolist()))
    flush = L2Flush(dev)
    n_marks = len(PHASES) + 1
    for _ in range(max(args.warmup, 3)):
        op(x, ids, w)
    op.check()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_marks)] for _ in range(args.steps)]
    for row in evs:
        for e in row:
            e.record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    for k in range(args.steps):
        flush()
        op.call_timed(x, ids, w, evs[k])
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clk = clocks.stop()
    seg = np.array([[evs[k][i].elapsed_time(evs[k][i + 1]) for i in range(n_marks - 1)] for k in range(args.steps)])
    total = seg.sum(axis=1)
    ms = allreduce_max(float(total.mean()), world)
    routed_all = allreduce_sum(float(routed), world)
    phase_ms = seg.mean(axis=0)

    # e2e through the op with pinned host buffers
    hx = x.cpu().pin_memory()
    hids = ids.cpu().pin_memory()
    hw = w.cpu().pin_memory()
    hout = torch.empty((x.shape[0], cfg.n_embd), dtype=torch.float32).pin_memory()
    dx, dids, dw = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(w)
    dout = torch.empty((x.shape[0], cfg.n_embd), dtype=torch.float32, device=dev)
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for k in range(args.warmup + args.steps):
        flush()
        if k >= args.warmup:
            e2e_ev[k - args.warmup][0].record()
        dx.copy_(hx, non_blocking=True)
        dids.copy_(hids, non_blocking=True)
        dw.copy_(hw, non_blocking=True)
        op(dx, dids, dw, out=dout)
        hout.copy_(dout, non_blocking=True)
        if k >= args.warmup:
            e2e_ev[k - args.warmup][1].record()
    torch.cuda.synchronize()
    e2e_ms = allreduce_max(statistics.mean(a.elapsed_time(b) for a, b in e2e_ev), world)
    ref_out = op(x, ids, w)
    torch.cuda.synchronize()
    # split-K sums are added in arrival order: the two runs agree to fp32 rounding
    ref_cpu = ref_out.cpu().double()
    e2e_rel = float(torch.linalg.vector_norm(hout.double() - ref_cpu) / torch.linalg.vector_norm(ref_cpu))
    assert e2e_rel <= 1e-6, f"e2e output differs from the device-resident run (rel {e2e_rel:.2e})"

    pk = peaks()
    x_bytes = x.numel() * x.element_size()
    out_bytes = x.shape[0] * cfg.n_embd * 4
    op_bytes = kind_bytes(es, KINDS, touched) + x_bytes + out_bytes
    dom = 1
    ach = op_bytes / (phase_ms[dom] * 1e-3) / 1e9
    op_ach = op_bytes / (total.mean() * 1e-3) / 1e9
    per_route_kernels = 1 if R <= 4096 else 3
    line = {
        "metric": METRIC, "value": routed_all / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE recipe)",
        "config": config_json(cfg, ids), "parallel": "single GPU",
        "roofline": {"bound": "hbm", "kernel": PHASES[dom], "achieved": ach, "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": ach / pk["hbm_gbs"], "traffic": None,
                     "algorithmic_bytes": op_bytes, "mean_ms": float(phase_ms[dom]),
                     "peak_source": pk["source"]},
        "roofline_op": {"achieved": op_ach, "frac": op_ach / pk["hbm_gbs"], "unit": "GB/s",
                        "algorithmic_bytes": op_bytes, "touched_experts": len(touched)},
        "phase_ms": {PHASES[i]: float(phase_ms[i]) for i in range(len(PHASES))},
        "e2e": {"value": routed_all / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hids.numel() * 4 + hw.numel() * 4),
                "d2h_bytes_per_step": int(hout.numel() * 4)},
        "gpu_launches": args.steps * (per_route_kernels + 1),
        "clocks": clk,
        "gen_s": gen_s,
    }
    if world == 1:
        line["router"] = run_router(dev, flush, steps=max(args.steps, 5), warmup=max(args.warmup, 3))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_leg(cfg, es, x, ids, w, args.cpu_seconds)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if world == 1 and args.config == 1 and not (args.no_prefill and args.no_sweep):
        del es, op
        torch.cuda.empty_cache()
        if not args.no_prefill:
            line["prefill"] = run_prefill(args, 2, dev, steps=max(5, min(args.steps, 20)), warmup=args.warmup)
            torch.cuda.empty_cache()
        if not args.no_sweep:
            line["sweep"] = run_sweep(dev, flush, steps=max(5, min(args.steps, 20)), warmup=max(args.warmup, 3))
    return line


SWEEP_POINTS = ((256, (1, 8, 64, 256)), (64, (64,)), (512, (64,)))


def run_sweep(dev, flush, steps: int, warmup: int):
    """Decode path on config 4's layer (256 experts, d 7168, f 2048, top-8) at several ranks and batch
    sizes: routed tokens/s and the whole op's algorithmic bytes (touched experts' factors + x + out)
    over its event time, against the HBM peak."""
    from latent_b200 import ExpertFFN, synth
    pk = peaks()
    out = []
    for rank, batches in SWEEP_POINTS:
        es = synth.make_expert_set(synth.sweep_config(rank, 1), device=dev)
        op = ExpertFFN(es, path="decode")
        for b in batches:
            cfg = synth.sweep_config(rank, b)
            x, ids, w = synth.make_batch(cfg, dev)
            for _ in range(warmup):
                op(x, ids, w)
            op.check()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            for a, e in ev:
                flush()
                a.record()
                op(x, ids, w)
                e.record()
            torch.cuda.synchronize()
            ms = statistics.mean(a.elapsed_time(e) for a, e in ev)
            touched = sorted(set(ids[ids >= 0].cpu().tolist()))
            nbytes = kind_bytes(es, KINDS, touched) + x.numel() * x.element_size() + x.shape[0] * cfg.n_embd * 4
            routed = int((ids >= 0).sum())
            out.append({"workload": cfg.name, "rank": rank, "tokens": b, "routed": routed,
                        "experts_touched": len(touched), "ms": ms, "value": routed / (ms * 1e-3), "unit": UNIT,
                        "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / (ms * 1e-3) / 1e9,
                        "frac_hbm": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]})
        del es, op
        torch.cuda.empty_cache()
    return out


def run_router(dev, flush, steps: int, warmup: int, T: int = 16384, E: int = 256, k: int = 8):
    """Adaptive top-k router (latent_router_topk) on config 3's routing shape, L2 flushed before each call."""
    from latent_b200 import router_topk
    g = torch.Generator(device=dev).manual_seed(3)
    scores = torch.softmax(torch.randn((T, E), generator=g, device=dev), dim=1)
    for _ in range(warmup):
        router_topk(scores, k)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev:
        flush()
        a.record()
        ids, w, nk = router_topk(scores, k)
        b.record()
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    nbytes = T * E * 4 + T * k * 8 + T * 4
    pk = peaks()
    return {"shape": {"tokens": T, "experts": E, "top_k": k, "threshold": 0.95}, "ms": ms,
            "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / (ms * 1e-3) / 1e9,
            "frac_hbm": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
            "mean_kept": float(nk.float().mean())}


PREFILL_PHASES = ["route", "dequant+gather", "G1 x.[A_g|A_u]", "G2 silu(t_g.B_g)*(t_u.B_u)", "G3 h.A_d",
                  "G4 s.B_d", "combine"]


def run_prefill(args, cfg_id: int, dev, steps: int, warmup: int):
    """Prefill leg (tcgen05 path): per-kernel CUDA-event times, tensor-core roofline."""
    from latent_b200 import ExpertFFN
    cfg, es, x, ids, w, gen_s = workload(cfg_id, dev, 0)
    op = ExpertFFN(es, path="prefill")
    flush = L2Flush(dev)
    for _ in range(max(warmup, 3)):
        op(x, ids, w)
    op.check()
    n_marks = len(PREFILL_PHASES) + 1
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_marks)] for _ in range(steps)]
    for row in evs:
        for e in row:
            e.record()
    torch.cuda.synchronize()
    for k in range(steps):
        flush()
        op.call_timed(x, ids, w, evs[k])
    torch.cuda.synchronize()
    seg = np.array([[evs[k][i].elapsed_time(evs[k][i + 1]) for i in range(n_marks - 1)] for k in range(steps)])
    phase_ms = seg.mean(axis=0)
    total = float(seg.sum(axis=1).mean())
    R = int((ids >= 0).sum())
    d, f, r = cfg.n_embd, cfg.n_ff, cfg.rank
    flops = {2: 2 * d * 2 * r * R, 3: 2 * r * 2 * f * R, 4: 2 * f * r * R, 5: 2 * r * d * R}
    dom = max(flops, key=lambda i: phase_ms[i])
    pk = peaks()
    ach = flops[dom] / (phase_ms[dom] * 1e-3) / 1e12
    all_flops = sum(flops.values())
    gemm_ms = float(sum(phase_ms[i] for i in flops))
    return {
        "workload": cfg.name, "value": R / (total * 1e-3), "unit": UNIT, "ms_per_step": total, "steps": steps,
        "routed": R, "dtype": "f16 MMA, f32 accumulate",
        "roofline": {"bound": "tensor", "kernel": PREFILL_PHASES[dom], "achieved": ach, "peak": pk["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": ach / pk["bf16_tflops"], "traffic": None, "flops": flops[dom],
                     "mean_ms": float(phase_ms[dom]), "peak_source": pk["source"] + " (burst bf16 GEMM)"},
        "roofline_gemms": {"achieved": all_flops / (gemm_ms * 1e-3) / 1e12, "flops": all_flops,
                           "frac": all_flops / (gemm_ms * 1e-3) / 1e12 / pk["bf16_tflops"], "unit": "TFLOP/s"},
        "roofline_step": {"achieved": all_flops / (total * 1e-3) / 1e12,
                          "frac": all_flops / (total * 1e-3) / 1e12 / pk["bf16_tflops"], "unit": "TFLOP/s"},
        "phase_ms": {PREFILL_PHASES[i]: float(phase_ms[i]) for i in range(len(PREFILL_PHASES))},
        # routing (1 or 3), tile offsets + 6 dequant + gather, 4 GEMMs (the combine runs in G4's epilogue)
        "gpu_launches": steps * ((1 if ids.numel() <= 4096 else 3) + 8 + 4),
        "gen_s": gen_s,
    }


class _TimedOps:
    """Wraps the EP ops to record events around the local fused FFN (the dominant kernel chain)."""

    def __init__(self, ops):
        self.ops = ops
        self.ev = None

    def dispatch(self, *a):
        return self.ops.dispatch(*a)

    def local_ffn(self, rx, lids, rw, wbd):
        if self.ev is not None:
            self.ev[0].record()
        y = self.ops.local_ffn(rx, lids, rw, wbd)
        if self.ev is not None:
            self.ev[1].record()
        return y

    def combine(self, *a):
        return self.ops.combine(*a)

    def __getattr__(self, name):   # the fixed-capacity pack/combine of the wrapped ops
        return getattr(self.ops, name)


def run_ours_ep(args, world, rank, local):
    """Expert-parallel step on `world` GPUs: experts sharded contiguously, a full config batch per rank
    (weak scaling), NCCL all-to-all dispatch and return."""
    from latent_b200 import ExpertSet, synth
    from latent_b200.ep import CudaEPOps, ExpertParallelFFN
    dev = torch.device("cuda", local)
    cfg = synth.CONFIGS[args.config]
    e_local = cfg.n_expert // world
    t0 = time.perf_counter()
    facs = synth.make_expert_factors(cfg, dev, experts=range(rank * e_local, (rank + 1) * e_local))
    es = ExpertSet(facs, device=dev, rank=cfg.rank)
    x, ids, w = synth.make_batch(cfg, dev, seed_offset=rank)
    gen_s = time.perf_counter() - t0
    ops = _TimedOps(CudaEPOps(es, cfg.n_expert))
    ep = ExpertParallelFFN(cfg.n_expert, ops, max_tokens=None if args.ep_exact else x.shape[0])
    flush = L2Flush(dev)
    for _ in range(max(args.warmup, 3)):
        ep(x, ids, w)
    torch.cuda.synchronize()
    step = lambda: ep(x, ids, w)
    graph = None
    if not args.ep_eager and not args.ep_exact:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                ep(x, ids, w)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        barrier(world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ep(x, ids, w)
        torch.cuda.synchronize()
        barrier(world)
        step = graph.replay
    steps = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    ffn = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    recv_rows = []
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    for k in range(args.steps):
        flush()
        ops.ev = None if graph is not None else ffn[k]
        steps[k][0].record()
        step()
        steps[k][1].record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ops.ev = None
    if graph is not None:
        # the local FFN alone, eagerly, for the roofline numerator's time
        for k in range(args.steps):
            flush()
            ops.ev = ffn[k]
            ep(x, ids, w)
        torch.cuda.synchronize()
        ops.ev = None
    recv_rows.append(sum(ep.last_counts[1]))
    ms_local = statistics.mean(a.elapsed_time(b) for a, b in steps)
    ffn_ms = statistics.mean(a.elapsed_time(b) for a, b in ffn)
    ms = allreduce_max(ms_local, world)
    routed = int((ids >= 0).sum())
    routed_all = allreduce_sum(float(routed), world)
    # every local expert receives rows at this batch size: the local FFN streams all of them
    local_bytes = es.factor_bytes(range(e_local))
    ach = local_bytes / (ffn_ms * 1e-3) / 1e9
    pk = peaks()
    # e2e with pinned host buffers
    hx, hids, hw = x.cpu().pin_memory(), ids.cpu().pin_memory(), w.cpu().pin_memory()
    hout = torch.empty((x.shape[0], cfg.n_embd), dtype=torch.float32).pin_memory()
    dx, dids, dw = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(w)
    e2e = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    e2e_graph = None
    if graph is not None:
        e2e_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(e2e_graph):
            e2e_out = ep(dx, dids, dw)
        torch.cuda.synchronize()
        barrier(world)
    for k in range(args.warmup + args.steps):
        flush()
        if k >= args.warmup:
            e2e[k - args.warmup][0].record()
        dx.copy_(hx, non_blocking=True)
        dids.copy_(hids, non_blocking=True)
        dw.copy_(hw, non_blocking=True)
        if e2e_graph is not None:
            e2e_graph.replay()
            out = e2e_out
        else:
            out = ep(dx, dids, dw)
        hout.copy_(out, non_blocking=True)
        if k >= args.warmup:
            e2e[k - args.warmup][1].record()
    torch.cuda.synchronize()
    e2e_ms = allreduce_max(statistics.mean(a.elapsed_time(b) for a, b in e2e), world)
    del graph, e2e_graph   # graphs holding NCCL work are released before the process group
    R = ids.numel()
    return {
        "metric": METRIC, "value": routed_all / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE recipe)",
        "config": config_json(cfg, ids),
        "parallel": (f"expert-parallel ep{world} (NCCL all-to-all, "
                     f"{'exact splits' if args.ep_exact else 'fixed capacity'}"
                     f"{', CUDA graph' if not args.ep_eager and not args.ep_exact else ''})"),
        "roofline": {"bound": "hbm", "kernel": "local fused expert FFN (rank 0)", "achieved": ach,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"], "traffic": None,
                     "algorithmic_bytes": local_bytes, "mean_ms": ffn_ms, "peak_source": pk["source"]},
        "e2e": {"value": routed_all / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hids.numel() * 4 + hw.numel() * 4),
                "d2h_bytes_per_step": int(hout.numel() * 4)},
        "gpu_launches": args.steps * ((1 if R <= 4096 else 3) + 1 + 2 + 1),
        "recv_rows_rank0": statistics.mean(recv_rows),
        "clocks": clk,
        "gen_s": gen_s,
    }


def run_reference(args, world, rank, local):
    if rank != 0:
        return None
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    cfg, es, x, ids, w, gen_s = workload(args.config, dev, 0)
    cb = cpu_leg(cfg, es, x, ids, w, seconds=0.0, min_steps=args.warmup + args.steps)
    value = cb["value"]
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE recipe)",
        "config": config_json(cfg, ids), "parallel": f"host CPU ({cb['cores']} threads)",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cb["cores"], "kind": "port", "sample": cb["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_only(args):
    """One leg alone on cuda:0 (profiling): the op runs warm-up + steps times, nothing else is timed."""
    dev = torch.device("cuda", 0)
    flush = L2Flush(dev)
    steps, warmup = args.steps, args.warmup
    if args.only == "router":
        return {"router": run_router(dev, flush, steps=steps, warmup=warmup)}
    if args.only == "prefill":
        return {"prefill": run_prefill(args, 2, dev, steps=steps, warmup=warmup)}
    if args.only == "sweep":
        return {"sweep": run_sweep(dev, flush, steps=steps, warmup=warmup)}
    from latent_b200 import ExpertFFN
    cfg, es, x, ids, w, _ = workload(args.config, dev, 0)
    op = ExpertFFN(es, path="decode")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for k in range(warmup + steps):
        flush()
        if k >= warmup:
            ev[k - warmup][0].record()
        op(x, ids, w)
        if k >= warmup:
            ev[k - warmup][1].record()
    op.check()
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    return {"decode": {"workload": cfg.name, "ms": ms, "value": int((ids >= 0).sum()) / (ms * 1e-3), "unit": UNIT}}


def main() -> int:
    args = parse_args()
    if args.only:
        torch.cuda.set_device(0)
        print(json.dumps(run_only(args)), flush=True)
        return 0
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank, local)
        elif world > 1:
            line = run_ours_ep(args, world, rank, local)
        else:
            line = run_ours(args, world, rank, local)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
