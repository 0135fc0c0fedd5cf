"""latent_expert_ffn_forward_noalloc: the entry point for callers that cannot
allocate device memory at call time (it uses the library's own fixed device
scratch instead of a caller workspace).  Checked through the C ABI against
the regular entry point, on two calls in a row with different batches, so
that state left in the shared scratch by one call cannot leak into the next.

Collected last on purpose: it must pass in a fresh process and after every
other test, and a failure here must not stop the rest of the suite.
"""

import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden
from gpu_helpers import golden_moe_experts
from latent_b200 import ExpertFFN, ExpertSet, synth
from latent_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _noalloc(op, x, ids, w):
    out = torch.full((x.shape[0], op.experts.n_embd), float("nan"), device=x.device)
    d = op.describe(x, ids, w, out)
    d.workspace, d.workspace_bytes = None, 0     # the caller provides no workspace
    st = _lib.lib().latent_expert_ffn_forward_noalloc(C.byref(d), torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.STATUS_NAMES.get(st, st)
    return out


@pytest.mark.parametrize("layer", ["golden", "c0"])
def test_noalloc_matches_regular_entry_on_consecutive_calls(cuda, layer):
    dev = torch.device("cuda", 0)
    if layer == "golden":
        z = golden("moe")
        facs, _ = golden_moe_experts(z)
        es = ExpertSet(facs, device=dev)
        batches = [(torch.from_numpy(z["x"]), torch.from_numpy(z["ids"]), torch.from_numpy(z["weights"]))]
        x2 = torch.from_numpy(z["x"][::-1].copy())
        batches.append((x2, torch.from_numpy(z["ids"][::-1].copy()), torch.from_numpy(z["weights"][::-1].copy())))
    else:
        cfg = synth.CONFIGS[0]
        es = ExpertSet(synth.make_expert_factors(cfg, "cpu"), device=dev, rank=cfg.rank)
        batches = [synth.make_batch(cfg, "cpu", seed_offset=s) for s in (11, 12)]
    op = ExpertFFN(es, path="decode")
    for x, ids, w in batches:                     # two calls in a row, different batches
        x, ids, w = x.to(dev), ids.to(dev), w.to(dev)
        ref = op(x, ids, w).clone()
        got = _noalloc(op, x, ids, w)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert O.rel_l2(ref.cpu().numpy(), got.cpu().numpy()) <= TOL


def test_noalloc_reports_device_errors(cuda):
    """A routed id past n_expert is skipped and recorded in the scratch's
    error word; latent_expert_ffn_check_noalloc reads it, and the next clean
    call clears it."""
    z = golden("moe")
    facs, _ = golden_moe_experts(z)
    es = ExpertSet(facs, device="cuda")
    op = ExpertFFN(es, path="decode")
    x = torch.from_numpy(z["x"]).cuda()
    ids = torch.from_numpy(z["ids"]).cuda()
    w = torch.from_numpy(z["weights"]).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    bad = ids.clone()
    bad[1, 0] = es.n_expert + 3
    out = torch.zeros((x.shape[0], es.n_embd), device="cuda")
    d = op.describe(x, bad, w, out)
    assert _lib.lib().latent_expert_ffn_forward_noalloc(C.byref(d), stream) == 0
    assert _lib.lib().latent_expert_ffn_check_noalloc(C.byref(d), stream) == 5   # LATENT_ERR_EXPERT_ID
    d = op.describe(x, ids, w, out)
    assert _lib.lib().latent_expert_ffn_forward_noalloc(C.byref(d), stream) == 0
    assert _lib.lib().latent_expert_ffn_check_noalloc(C.byref(d), stream) == 0


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    z = golden("moe")
    facs, _ = golden_moe_experts(z)
    es = ExpertSet(facs, device="cuda")
    op = ExpertFFN(es, path="decode")
    d = op.describe(torch.zeros((2, es.n_embd), device="cuda"), torch.zeros((2, 2), dtype=torch.int32, device="cuda"),
                    torch.zeros((2, 2), device="cuda"), torch.zeros((2, es.n_embd), device="cuda"))
    d.n_tokens = 1 << 20                          # needs far more than 16 MiB of scratch
    st = _lib.lib().latent_expert_ffn_forward_noalloc(C.byref(d), torch.cuda.current_stream().cuda_stream)
    assert st == 6                                # LATENT_ERR_WORKSPACE, nothing queued
