"""Dense-fallback experts on the GPU.

The reference compressor stores `<name>.dense_fallback` (fp16) when a
matrix's factors miss the error threshold (loader/latent_loader.py:262-265);
the dense expert forward is dense_swiglu_expert (loader/latent_runtime.py:
62-73).  A mixed routed batch -- latent experts through the fused op, flagged
experts through the dense kernels, one of them dense in every kind, two of
them dense in one kind only -- is checked against a numpy restatement that
applies, per routed slot, the dense matrix of a flagged kind and the factor
pair of every other kind, then the top-k combine.  Tolerance rel-L2 <= 1e-5
(fp32 accumulation on both sides).
"""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_helpers import oracle_experts, rel
from latent_b200 import ExpertFFN, ExpertSet, synth
from latent_b200 import runtime as L

pytestmark = pytest.mark.gpu
TOL = 1e-5
FLAGGED = {1: ("gate", "up", "down"), 3: ("down",), 6: ("gate",)}


def _dense_matrices(pairs, kinds, seed):
    """fp16 dense copies near A @ B (perturbed, so that using them is visible)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name in kinds:
        a, b = pairs[("gate", "up", "down").index(name)]
        w = a @ b
        w = w + 0.05 * np.abs(w).mean() * rng.standard_normal(w.shape).astype(np.float32)
        out[name] = w.astype(np.float16)
    return out


def _reference(x, ids, w, pairs, dense, wbd, per_slot):
    T, k = ids.shape
    d = x.shape[1]
    out = np.zeros((T, k, d) if per_slot else (T, d), np.float64)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            if e < 0:
                continue
            proj = []
            for m, name in enumerate(("gate", "up", "down")):
                if name in dense.get(e, {}):
                    proj.append(lambda v, W=dense[e][name].astype(np.float32): v @ W)
                else:
                    proj.append(lambda v, P=pairs[e][m]: (v @ P[0]) @ P[1])
            xv = x[t:t + 1].astype(np.float32)
            h = O.silu(proj[0](xv)) * proj[1](xv)
            if wbd:
                h = h * np.float32(w[t, j])
            y = proj[2](h)[0].astype(np.float64)
            if per_slot:
                out[t, j] = y
            else:
                out[t] += (1.0 if wbd else float(w[t, j])) * y
    return out


@pytest.fixture(scope="module")
def layer(cuda):
    cfg = synth.CONFIGS[0]
    facs = synth.make_expert_factors(cfg, "cpu")
    pairs = oracle_experts(facs, rank=cfg.rank)
    dense = {e: _dense_matrices(pairs[e], kinds, 100 + e) for e, kinds in FLAGGED.items()}
    es = ExpertSet(facs, device="cuda", rank=cfg.rank, dense=dense)
    return cfg, es, pairs, dense


@pytest.mark.parametrize("wbd", [False, True])
@pytest.mark.parametrize("per_slot", [False, True])
@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_mixed_latent_and_dense_batch(layer, wbd, per_slot, path):
    cfg, es, pairs, dense = layer
    x, ids, w = synth.make_batch(cfg, "cpu", seed_offset=3)
    ids[0, 1] = -1                                 # a skipped slot
    ids[5] = torch.tensor([1, 3], dtype=torch.int32)   # flagged experts on one token
    flagged = np.isin(ids.numpy(), list(FLAGGED)).sum()
    assert flagged > 4 and (ids.numpy() >= 0).sum() - flagged > 4
    y = ExpertFFN(es, path=path)(x.cuda(), ids.cuda(), w.cuda(), weight_before_down=wbd, out_per_slot=per_slot)
    ref = _reference(x.numpy(), ids.numpy(), w.numpy(), pairs, dense, wbd, per_slot)
    assert rel(ref, y) <= (TOL if path == "decode" else 2e-3)


def test_dense_only_batch_and_empty_batch(layer):
    cfg, es, pairs, dense = layer
    x, ids, w = synth.make_batch(cfg, "cpu", n_tokens=9, seed_offset=4)
    ids[:] = torch.tensor([1, 6], dtype=torch.int32)
    y = ExpertFFN(es, path="decode")(x.cuda(), ids.cuda(), w.cuda())
    assert rel(_reference(x.numpy(), ids.numpy(), w.numpy(), pairs, dense, False, False), y) <= TOL
    e = ExpertFFN(es)(torch.zeros((0, cfg.n_embd), device="cuda"), torch.zeros((0, 2), dtype=torch.int32,
                      device="cuda"), torch.zeros((0, 2), device="cuda"))
    assert e.shape == (0, cfg.n_embd)


def test_dense_swiglu_expert_and_project_use_the_library_kernel(layer):
    cfg, es, pairs, dense = layer
    rng = np.random.default_rng(8)
    x = rng.standard_normal((5, cfg.n_embd)).astype(np.float32)
    g, u, dn = (dense[1][n] for n in ("gate", "up", "down"))
    want = O.dense_swiglu_expert(x, g.astype(np.float32), u.astype(np.float32), dn.astype(np.float32))
    assert O.rel_l2(want, L.dense_swiglu_expert(x, g, u, dn)) <= TOL
    # odd shapes go through the same kernel (zero padding)
    a = rng.standard_normal((7, 37)).astype(np.float32)
    b = rng.standard_normal((37, 5)).astype(np.float32)
    got = L._matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert O.rel_l2(a @ b, got) <= 1e-6


def test_load_pair_reads_dense_fallback_on_request(cuda):
    """Reference NPZ arrays (tests/golden/runtime.npz) plus a `<name>.dense_fallback` key."""
    from conftest import golden
    z = golden("runtime")
    arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith("nf4/")}
    x = arrays["x"]
    a, b = O.pair_from_npz(arrays, "gate")
    dense = (a @ b + 0.1).astype(np.float16)
    arrays["gate.dense_fallback"] = dense
    plain = L.load_pair(arrays, "gate")                   # the reference behaviour: fallback ignored
    assert plain.dense is None
    assert O.rel_l2(O.project(x, a, b), L.project(x, plain)) <= TOL
    served = L.load_pair(arrays, "gate", dense_fallback=True)
    assert O.rel_l2(x.astype(np.float32) @ dense.astype(np.float32), L.project(x, served)) <= 1e-6
