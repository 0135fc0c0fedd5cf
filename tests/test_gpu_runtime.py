"""The reference-API mirror (latent_b200.runtime) on the GPU, read like the
reference's own runtime tests (tests/test_latent_loader.py:100-141) but
pinned to the reference's recorded outputs at fp32 tolerance."""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden
import latent_b200 as L

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _arrays(variant):
    z = golden("runtime")
    return z, {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(variant + "/")}


@pytest.mark.parametrize("variant", ["nf4", "int8"])
def test_swiglu_expert_matches_reference_output(cuda, variant):
    z, arrays = _arrays(variant)
    gate, up, down = (L.load_pair(arrays, n) for n in ("gate", "up", "down"))
    y = L.swiglu_expert(arrays["x"], gate, up, down)
    assert isinstance(y, np.ndarray) and y.shape == arrays["y"].shape
    assert O.rel_l2(arrays["y"], y) <= TOL
    y2 = L.swiglu_expert(arrays["x"], gate, up, down, weight=0.3, weight_before_down=True)
    assert O.rel_l2(arrays["y_wbd"], y2) <= TOL


def test_weight_before_down_equals_post_scaling(cuda):
    z, arrays = _arrays("nf4")
    gate, up, down = (L.load_pair(arrays, n) for n in ("gate", "up", "down"))
    before = L.swiglu_expert(arrays["x"], gate, up, down, weight=0.25, weight_before_down=True)
    after = L.swiglu_expert(arrays["x"], gate, up, down) * 0.25
    assert np.allclose(before, after, rtol=1e-5, atol=1e-7)


def test_missing_factor_raises_keyerror(cuda):
    _, arrays = _arrays("nf4")
    del arrays["gate.b.nf4"]
    with pytest.raises(KeyError):
        L.load_pair(arrays, "gate")


def test_silu_project_and_dense(cuda):
    z, arrays = _arrays("nf4")
    x = np.linspace(-30, 30, 1001, dtype=np.float32)
    assert O.rel_l2(O.silu(x), L.silu(x)) <= 1e-6
    pair = L.load_pair(arrays, "gate")
    ref = O.project(arrays["x"], *O.pair_from_npz(arrays, "gate"))
    assert O.rel_l2(ref, L.project(arrays["x"], pair)) <= TOL
    dense = [z[f"dense/{n}"] for n in ("gate", "up", "down")]
    assert O.rel_l2(arrays["dense_y"], L.dense_swiglu_expert(arrays["x"], *dense)) <= TOL


def test_moe_expert_ffn_numpy_roundtrip(cuda):
    from gpu_helpers import golden_moe_experts
    z = golden("moe")
    facs, _ = golden_moe_experts(z)
    es = L.ExpertSet(facs, device="cuda")
    out = L.moe_expert_ffn(z["x"], z["ids"], z["weights"], es)
    assert isinstance(out, np.ndarray)
    assert O.rel_l2(z["out"], out) <= TOL
