"""The CPU oracle against the golden vectors recorded from the reference runtime.

These pin the oracle: every byte the reference's encoders produce and every
value its decoders return must come out of the oracle bit for bit; the
SwiGLU outputs agree to fp32 round-off (both sides run numpy fp32 GEMMs).
"""

import numpy as np
import pytest

import oracle as O
from conftest import golden


def test_nf4_encode_decode_bit_exact():
    z = golden("nf4")
    for i in range(int(z["n_cases"])):
        v, g = z[f"c{i}.values"], int(z[f"c{i}.group"])
        packed, scales, shape = O.nf4_encode(v, g)
        assert np.array_equal(packed, z[f"c{i}.packed"]), i
        assert np.array_equal(scales.view(np.uint16), z[f"c{i}.scales"].view(np.uint16)), i
        assert tuple(shape) == tuple(z[f"c{i}.shape"])
        dec = O.nf4_decode(z[f"c{i}.packed"], z[f"c{i}.scales"], shape, g)
        assert np.array_equal(dec.view(np.uint32), z[f"c{i}.decoded"].view(np.uint32)), i


def test_int8_encode_decode_bit_exact():
    z = golden("int8")
    for i in range(int(z["n_cases"])):
        v, g = z[f"c{i}.values"], int(z[f"c{i}.group"])
        q, scales, shape = O.int8_encode(v, g)
        assert np.array_equal(q, z[f"c{i}.q"]), i
        assert np.array_equal(scales.view(np.uint16), z[f"c{i}.scales"].view(np.uint16)), i
        dec = O.int8_decode(z[f"c{i}.q"], z[f"c{i}.scales"], shape, g)
        assert np.array_equal(dec.view(np.uint32), z[f"c{i}.decoded"].view(np.uint32)), i


def test_mixed_groups_match_reference_encoders():
    z = golden("mixed")
    enc = O.mixed_encode(z["values"], snr_db=20.0)
    assert np.array_equal(enc["is_int8"], z["is_int8"])
    assert 0 < enc["is_int8"].sum() < enc["is_int8"].size
    assert np.array_equal(enc["nf4"], z["nf4"])
    assert np.array_equal(enc["scales"].view(np.uint16), z["scales"].view(np.uint16))
    assert np.array_equal(enc["int8"], z["int8"])
    dec = O.mixed_decode(enc)
    assert np.array_equal(dec.view(np.uint32), z["decoded"].view(np.uint32))


@pytest.mark.parametrize("variant", ["nf4", "int8"])
def test_runtime_swiglu_matches_reference(variant):
    z = golden("runtime")
    arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(variant + "/")}
    pairs = [O.pair_from_npz(arrays, n) for n in ("gate", "up", "down")]
    y = O.swiglu_expert(arrays["x"], *pairs)
    assert O.rel_l2(arrays["y"], y) < 1e-6
    y2 = O.swiglu_expert(arrays["x"], *pairs, weight=0.3, weight_before_down=True)
    assert O.rel_l2(arrays["y_wbd"], y2) < 1e-6
    dense = [z[f"dense/{n}"] for n in ("gate", "up", "down")]
    assert O.rel_l2(arrays["dense_y"], O.dense_swiglu_expert(arrays["x"], *dense)) < 1e-6


def test_runtime_missing_factor_raises_keyerror():
    z = golden("runtime")
    arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith("nf4/") and ".nf4" not in k}
    with pytest.raises(KeyError):
        O.pair_from_npz(arrays, "gate")


@pytest.mark.parametrize("wbd", [False, True])
def test_moe_forward_matches_reference_combine(wbd):
    z = golden("moe")
    E = int(z["E"])
    experts = []
    for e in range(E):
        arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(f"e{e}/")}
        experts.append(tuple(O.pair_from_npz(arrays, n) for n in ("gate", "up", "down")))
    out = O.moe_forward(z["x"], z["ids"], z["weights"], experts, weight_before_down=wbd)
    assert O.rel_l2(z["out_wbd" if wbd else "out"], out) < 1e-6
    per_slot = O.moe_forward(z["x"], z["ids"], z["weights"], experts, weight_before_down=wbd, out_per_slot=True)
    assert O.rel_l2(z["per_slot_wbd" if wbd else "per_slot"], per_slot) < 1e-6
    # skipped slots give exact zero rows
    assert not per_slot[z["ids"] < 0].any()


def test_route_is_stable_and_skips_negative_ids():
    ids = np.array([[2, 0], [2, -1], [0, 2], [1, 1]], np.int32)
    counts, offsets, order = O.route(ids, 4)
    assert counts.tolist() == [2, 2, 3, 0]
    assert offsets.tolist() == [0, 2, 4, 7, 7]
    assert order.tolist() == [1, 4, 6, 7, 0, 2, 5]


def test_router_topk_matches_reference_adaptive_topk():
    """oracle.router_topk vs adaptive_topk_batch (loader/adaptive_topk.py:59-90) on recorded cases."""
    z = golden("router")
    for c in range(int(z["n_cases"])):
        scores, k, th = z[f"c{c}/scores"], int(z[f"c{c}/top_k"]), float(z[f"c{c}/threshold"])
        ids, w, n_kept = O.router_topk(scores, k, th)
        assert np.array_equal(n_kept, z[f"c{c}/n_kept"]), c
        keep = z[f"c{c}/keep"]
        assert np.array_equal(ids >= 0, keep), c
        assert np.array_equal(ids[keep], z[f"c{c}/order"][keep]), c
        live = n_kept > 0
        assert np.allclose(w[live].sum(axis=1), 1.0, atol=1e-6)
        assert not w[~keep].any()


def test_router_topk_validates_like_reference():
    with pytest.raises(ValueError):
        O.router_topk(np.ones((2, 4), np.float32), 2, threshold=0.0)
    with pytest.raises(ValueError):
        O.router_topk(np.ones((2, 4), np.float32), 5)
