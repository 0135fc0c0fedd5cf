"""Parity at the benchmark configurations' full shapes.

- config 2 (the prefill bench: 8 experts, d 4096, f 14336, rank 512, 4% of
  columns outliers so some groups fall back to INT8): the full 8192-token
  prefill, a 512-token sample spread over the batch (every expert, rows on
  both sides of the 128-row MMA tiles) against the numpy oracle; and the
  decode path at rank 512 on 32 tokens.
- configs 3/4 shapes (256 experts, d 7168, f 2048, top-8) at ranks 64 and 512:
  decode on 64 tokens and prefill on 4096 tokens (Zipf-skewed routing), a
  token sample against the reference.
(config 1, the decode bench, is checked on its whole batch in
tests/test_gpu_fullsize.py.)

For configs 1-2 the oracle decodes the factors itself (oracle.decode_grouped).
The 256-expert layers are too large for that to finish in seconds, so their
reference forward (loader/latent_runtime.py:48-59 plus the top-k combine) is
evaluated in float64 on the GPU, expert by expert, from factors dequantized by
latent_dequantize, which tests/test_gpu_decode.py pins bit-exact to the
reference decoder.  Tolerances: rel-L2 <= 1e-5 (decode, fp32) and <= 2e-3
(prefill, 16-bit MMA operands).
"""

import pytest
import torch

import oracle as O
from gpu_helpers import decode, rel
from latent_b200 import ExpertFFN, dequantize, synth

pytestmark = pytest.mark.gpu
TOL_DECODE, TOL_PREFILL = 1e-5, 2e-3
KINDS = ("gate_a", "gate_b", "up_a", "up_b", "down_a", "down_b")


def _expert_pairs(es, e):
    """((A_g, B_g), (A_u, B_u), (A_d, B_d)) of expert e, decoded by the oracle."""
    return tuple((decode(es[f"{n}_a"].expert(e)), decode(es[f"{n}_b"].expert(e))) for n in ("gate", "up", "down"))


def _oracle(es, n_expert, x, ids, w, **kw):
    ids_np = ids.cpu().numpy()
    touched = sorted(set(ids_np[ids_np >= 0].tolist()))
    table = [None] * n_expert
    for e in touched:
        table[e] = _expert_pairs(es, e)
    return O.moe_forward(x.float().cpu().numpy(), ids_np, w.float().cpu().numpy(), table, **kw)


def _reference_f64(es, x, ids, w):
    """The reference's routed SwiGLU + top-k combine in float64 on the GPU."""
    out = torch.zeros((x.shape[0], es.n_embd), dtype=torch.float64, device=x.device)
    xd = x.double()
    for e in torch.unique(ids[ids >= 0]).tolist():
        tok, slot = torch.nonzero(ids == e, as_tuple=True)
        f = {k: dequantize(es[k], e).double() for k in KINDS}
        xe = xd[tok]
        g = (xe @ f["gate_a"]) @ f["gate_b"]
        u = (xe @ f["up_a"]) @ f["up_b"]
        h = g / (1.0 + torch.exp(-g)) * u
        y = (h @ f["down_a"]) @ f["down_b"]
        out.index_add_(0, tok, y * w[tok, slot].double()[:, None])
    return out.cpu().numpy()


@pytest.fixture(scope="module")
def c2(cuda):
    cfg = synth.CONFIGS[2]
    return cfg, synth.make_expert_set(cfg, device="cuda")


def test_c2_full_prefill_token_sample(c2):
    cfg, es = c2
    x, ids, w = synth.make_batch(cfg, "cuda")
    y = ExpertFFN(es, path="prefill")(x, ids, w)
    sample = torch.arange(0, cfg.n_tokens, cfg.n_tokens // 512, device="cuda")[:512]
    xs, ids_s, ws = x[sample], ids[sample], w[sample]
    assert set(ids_s.flatten().tolist()) == set(range(cfg.n_expert))
    assert sum(es[k].n_int8 for k in KINDS) > 0, "config 2 is meant to carry INT8 groups"
    ref = _oracle(es, cfg.n_expert, xs, ids_s, ws)
    assert rel(ref, y[sample]) <= TOL_PREFILL


def test_c2_rank512_decode(c2):
    cfg, es = c2
    x, ids, w = synth.make_batch(cfg, "cuda", n_tokens=32, seed_offset=9)
    for wbd in (False, True):
        y = ExpertFFN(es, path="decode")(x, ids, w, weight_before_down=wbd)
        ref = _oracle(es, cfg.n_expert, x, ids, w, weight_before_down=wbd)
        assert rel(ref, y) <= TOL_DECODE, wbd


@pytest.mark.parametrize("rank", [64, 512])
def test_v3_shape_decode_and_prefill(cuda, rank):
    base = synth.sweep_config(rank, 64)
    es = synth.make_expert_set(base, device="cuda")
    # decode: the sweep's 64-token batch (~222 experts touched)
    x, ids, w = synth.make_batch(base, "cuda")
    y = ExpertFFN(es, path="decode")(x, ids, w)
    assert rel(_reference_f64(es, x, ids, w), y) <= TOL_DECODE
    # prefill: 4096 tokens with config 3's Zipf-skewed router, 256 sampled tokens
    pcfg = synth.CONFIGS[3].__class__(**{**base.__dict__, "zipf": 1.1, "n_tokens": 4096})
    x, ids, w = synth.make_batch(pcfg, "cuda", seed_offset=1)
    y = ExpertFFN(es, path="prefill")(x, ids, w)
    sample = torch.arange(0, 4096, 16, device="cuda")
    ref = _reference_f64(es, x[sample], ids[sample], w[sample])
    assert rel(ref, y[sample]) <= TOL_PREFILL
