"""GPU parity of the prefill path (tcgen05 f16 MMA, fp32 accumulate) against
the CPU oracle.  Tolerance: relative L2 <= 2e-3 (the north-star bound for the
16-bit-MMA path)."""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden
from gpu_helpers import decode, golden_moe_experts, oracle_experts, rel
from latent_b200 import ExpertFFN, ExpertSet, synth

pytestmark = pytest.mark.gpu
TOL = 2e-3


def test_golden_moe_layer_prefill(cuda):
    z = golden("moe")
    facs, _ = golden_moe_experts(z)
    es = ExpertSet(facs, device="cuda")
    op = ExpertFFN(es, path="prefill")
    args = [torch.from_numpy(z[k]).cuda() for k in ("x", "ids", "weights")]
    for wbd, per_slot in ((False, False), (True, False), (False, True)):
        y = op(*args, weight_before_down=wbd, out_per_slot=per_slot)
        key = ("per_slot" if per_slot else "out") + ("_wbd" if wbd else "")
        assert rel(z[key], y) <= TOL, key
    op.check()


@pytest.fixture(scope="module")
def c0(cuda):
    cfg = synth.CONFIGS[0]
    facs = synth.make_expert_factors(cfg, "cpu")
    return cfg, ExpertSet(facs, device="cuda", rank=cfg.rank), oracle_experts(facs)


@pytest.mark.parametrize("x_dtype", [torch.float32, torch.bfloat16])
def test_c0_prefill_matches_oracle(c0, x_dtype):
    cfg, es, ref_ex = c0
    x, ids, w = synth.make_batch(cfg, "cpu", n_tokens=600)   # ~150 rows per expert: several M tiles
    x = x.to(x_dtype)
    ref = O.moe_forward(x.float().numpy(), ids.numpy(), w.numpy(), ref_ex)
    y = ExpertFFN(es, path="prefill")(x.cuda(), ids.cuda(), w.cuda())
    assert rel(ref, y) <= TOL


def test_prefill_skewed_and_skipped_slots(c0):
    cfg, es, ref_ex = c0
    x, ids, w = synth.make_batch(cfg, "cpu", n_tokens=300, seed_offset=3)
    ids[:200, 0] = 5                 # one expert with 200+ rows, others sparse
    ids[::7, 1] = -1
    ref = O.moe_forward(x.numpy(), ids.numpy(), w.numpy(), ref_ex)
    y = ExpertFFN(es, path="prefill")(x.cuda(), ids.cuda(), w.cuda())
    assert rel(ref, y) <= TOL


def test_prefill_and_decode_agree(c0):
    cfg, es, _ = c0
    x, ids, w = (t.cuda() for t in synth.make_batch(cfg, "cpu", n_tokens=256, seed_offset=4))
    yp = ExpertFFN(es, path="prefill")(x, ids, w)
    yd = ExpertFFN(es, path="decode")(x, ids, w)
    assert rel(yd.cpu().numpy(), yp) <= TOL


def test_prefill_deterministic(c0):
    cfg, es, _ = c0
    x, ids, w = (t.cuda() for t in synth.make_batch(cfg, "cpu", n_tokens=512, seed_offset=5))
    op = ExpertFFN(es, path="prefill")
    a = op(x, ids, w).clone()
    b = op(x, ids, w)
    assert torch.equal(a, b)
