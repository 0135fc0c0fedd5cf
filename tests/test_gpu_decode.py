"""GPU parity of the decode path (fp32 CUDA-core chain) against the CPU oracle.

Tolerance: relative L2 <= 1e-5 against the fp32 reference runtime semantics
(oracle.moe_forward / swiglu_expert on the identical decoded factors);
dequantization is compared bit for bit.
"""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden
from gpu_helpers import decode, golden_moe_experts, oracle_experts, rel
from latent_b200 import ExpertFFN, ExpertSet, dequantize, quantize_factor, synth
from latent_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def dev(cuda):
    return torch.device("cuda", 0)


def test_dequant_bit_exact_reference_factors(dev):
    z = golden("runtime")
    from latent_b200 import format as F
    for variant in ("nf4", "int8"):
        arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(variant + "/")}
        for name in ("gate", "up", "down"):
            for side in ("a", "b"):
                gf = F.from_npz(arrays, name, side).to(dev)
                got = dequantize(gf).cpu().numpy()
                ref = O.factor_from_npz(arrays, name, side)
                assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (variant, name, side)


def test_dequant_bit_exact_mixed_groups(dev):
    rng = np.random.default_rng(21)
    v = rng.standard_normal((96, 256)).astype(np.float32)
    v[:, 11] *= 40.0
    v[3] = 0.0
    gf = quantize_factor(torch.from_numpy(v), 20.0)
    assert gf.n_int8 > 0
    got = dequantize(gf.to(dev)).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), decode(gf).view(np.uint32))


@pytest.mark.parametrize("wbd", [False, True])
@pytest.mark.parametrize("per_slot", [False, True])
def test_golden_moe_layer(dev, wbd, per_slot):
    z = golden("moe")
    facs, _ = golden_moe_experts(z)
    es = ExpertSet(facs, device=dev)
    op = ExpertFFN(es, path="decode")
    x = torch.from_numpy(z["x"]).to(dev)
    ids = torch.from_numpy(z["ids"]).to(dev)
    w = torch.from_numpy(z["weights"]).to(dev)
    y = op(x, ids, w, weight_before_down=wbd, out_per_slot=per_slot)
    key = ("per_slot" if per_slot else "out") + ("_wbd" if wbd else "")
    assert rel(z[key], y) <= TOL
    if per_slot:
        assert not y.cpu().numpy()[z["ids"] < 0].any()
    op.check()


@pytest.fixture(scope="module")
def c0(dev):
    cfg = synth.CONFIGS[0]
    facs = synth.make_expert_factors(cfg, "cpu")
    es = ExpertSet(facs, device=dev, rank=cfg.rank)
    return cfg, facs, es, oracle_experts(facs)


@pytest.mark.parametrize("x_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_c0_layer_matches_oracle(dev, c0, x_dtype):
    cfg, facs, es, ref_ex = c0
    x, ids, w = synth.make_batch(cfg, "cpu")
    x = x.to(x_dtype)
    ref = O.moe_forward(x.float().numpy(), ids.numpy(), w.numpy(), ref_ex)
    y = ExpertFFN(es, path="decode")(x.to(dev), ids.to(dev), w.to(dev))
    assert rel(ref, y) <= TOL


def test_c0_has_int8_groups_and_fp16_router_weights(dev, c0):
    cfg, facs, es, ref_ex = c0
    x, ids, w = synth.make_batch(cfg, "cpu", seed_offset=5)
    w16 = w.half()
    ref = O.moe_forward(x.numpy(), ids.numpy(), w16.float().numpy(), ref_ex, weight_before_down=True)
    y = ExpertFFN(es, path="decode")(x.to(dev), ids.to(dev), w16.to(dev), weight_before_down=True)
    assert rel(ref, y) <= TOL


def test_skewed_routing_one_expert_many_tokens(dev, c0):
    cfg, facs, es, ref_ex = c0
    x, ids, w = synth.make_batch(cfg, "cpu", n_tokens=37)
    ids[:, 0] = 3               # 37 tokens on expert 3: several 4-token chunks
    ids[::3, 1] = -1            # skipped slots
    ids[1, 1] = 0
    ref = O.moe_forward(x.numpy(), ids.numpy(), w.numpy(), ref_ex)
    y = ExpertFFN(es, path="decode")(x.to(dev), ids.to(dev), w.to(dev))
    assert rel(ref, y) <= TOL


def test_top1_and_single_token(dev, c0):
    cfg, facs, es, ref_ex = c0
    x, ids, w = synth.make_batch(cfg, "cpu", n_tokens=1)
    ids1, w1 = ids[:, :1].contiguous(), torch.ones((1, 1))
    ref = O.moe_forward(x.numpy(), ids1.numpy(), w1.numpy(), ref_ex)
    y = ExpertFFN(es, path="decode")(x.to(dev), ids1.to(dev), w1.to(dev))
    assert rel(ref, y) <= TOL


def test_empty_batch_is_noop(dev, c0):
    cfg, facs, es, _ = c0
    op = ExpertFFN(es, path="decode")
    y = op(torch.zeros((0, cfg.n_embd), device=dev), torch.zeros((0, 2), dtype=torch.int32, device=dev),
           torch.zeros((0, 2), device=dev))
    assert y.shape == (0, cfg.n_embd)


def test_out_of_range_expert_id_is_reported(dev, c0):
    cfg, facs, es, ref_ex = c0
    x, ids, w = synth.make_batch(cfg, "cpu", n_tokens=8)
    ids[2, 0] = cfg.n_expert + 5
    op = ExpertFFN(es, path="decode")
    y = op(x.to(dev), ids.to(dev), w.to(dev))
    with pytest.raises(_lib.LatentError) as ei:
        op.check()
    assert ei.value.status == 5
    ids_ref = ids.clone()
    ids_ref[2, 0] = -1         # the bad slot is skipped
    ref = O.moe_forward(x.numpy(), ids_ref.numpy(), w.numpy(), ref_ex)
    assert rel(ref, y) <= TOL


def test_repeat_calls_agree(dev, c0):
    """Split-K partial sums are added in arrival order: repeated calls agree
    to fp32 rounding of those sums, not bitwise."""
    cfg, facs, es, _ = c0
    x, ids, w = (t.to(dev) for t in synth.make_batch(cfg, "cpu"))
    op = ExpertFFN(es, path="decode")
    a = op(x, ids, w).clone()
    for _ in range(3):
        assert rel(a.cpu().numpy(), op(x, ids, w)) <= 1e-6
