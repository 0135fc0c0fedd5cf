"""The decode path at the benchmark's full size (config 1: 64 experts,
d=2048, f=1408, r=256, top-6, 32 tokens, bf16 activations): the whole batch
against the oracle, plus size-independent properties."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_helpers import decode, rel
from latent_b200 import ExpertFFN, synth

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def c1(cuda):
    cfg = synth.CONFIGS[1]
    es = synth.make_expert_set(cfg, device="cuda")
    x, ids, w = synth.make_batch(cfg, "cuda")
    return cfg, es, x, ids, w


def _oracle_experts(es, experts):
    out = {}
    for e in experts:
        out[e] = tuple((decode(es[f"{n}_a"].expert(e)), decode(es[f"{n}_b"].expert(e))) for n in ("gate", "up", "down"))
    return out


@pytest.mark.parametrize("wbd", [False, True])
def test_whole_batch_matches_oracle(c1, wbd):
    cfg, es, x, ids, w = c1
    y = ExpertFFN(es, path="decode")(x, ids, w, weight_before_down=wbd).cpu().numpy()
    ids_np = ids.cpu().numpy()
    ex = _oracle_experts(es, sorted(set(ids_np.ravel().tolist())))
    table = [ex.get(e) for e in range(cfg.n_expert)]
    ref = O.moe_forward(x.float().cpu().numpy(), ids_np, w.cpu().numpy(), table, weight_before_down=wbd)
    assert rel(ref, y) <= TOL


def test_weight_scaling_is_linear(c1):
    """Doubling the router weights doubles the output (exact in fp32 up to
    the arrival order of the split-K sums)."""
    cfg, es, x, ids, w = c1
    op = ExpertFFN(es, path="decode")
    y1 = op(x, ids, w).clone()
    y2 = op(x, ids, w * 2.0)
    assert rel((y1 * 2.0).cpu().numpy(), y2) <= 1e-6


def test_token_permutation_is_equivariant(c1):
    """Permuting tokens permutes the output, to fp32 rounding: the split-K
    partial sums are added in arrival order, and under a permutation an
    expert's tokens may be grouped into different 4-token virtual experts."""
    cfg, es, x, ids, w = c1
    op = ExpertFFN(es, path="decode")
    y = op(x, ids, w).clone()
    assert rel(y.cpu().numpy(), op(x, ids, w)) <= 1e-6
    perm = torch.randperm(x.shape[0], generator=torch.Generator().manual_seed(9)).to(x.device)
    yp = op(x[perm].contiguous(), ids[perm].contiguous(), w[perm].contiguous())
    assert rel(y[perm].cpu().numpy(), yp) <= 1e-6


def test_per_slot_rows_sum_to_combined(c1):
    cfg, es, x, ids, w = c1
    op = ExpertFFN(es, path="decode")
    y = op(x, ids, w).clone()
    ps = op(x, ids, w, out_per_slot=True)
    comb = (ps.double() * w.double()[:, :, None]).sum(dim=1)
    assert rel(comb.cpu().numpy(), y) <= 1e-6
