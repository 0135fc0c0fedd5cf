"""A LATENT GGUF layer loaded onto the GPU (latent_b200.gguf_io.load_layer)
runs the fused op with the reference's results: factors dequantize bit for
bit to the reference's values, the routed forward is within rel-L2 1e-5 of the
reference swiglu_expert outputs combined in fp64."""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN, golden
from latent_b200 import ExpertFFN, dequantize, gguf_io

pytestmark = pytest.mark.gpu
pytest.importorskip("gguf")


def test_gguf_layer_forward_matches_reference(cuda):
    z = golden("gguf_layer")
    es = gguf_io.load_layer(GOLDEN / "latent_layer.gguf", int(z["layer"]), device=torch.device("cuda", 0))
    for e in range(int(z["E"])):
        for kind in ("gate", "up", "down"):
            for side in ("a", "b"):
                want = z[f"e{e}/{kind}_{side}"]
                got = dequantize(es[f"{kind}_{side}"], e).cpu().numpy()[: want.shape[0], : want.shape[1]]
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (e, kind, side)
    dev = torch.device("cuda", 0)
    y = ExpertFFN(es, path="decode")(torch.from_numpy(z["x"]).to(dev), torch.from_numpy(z["ids"]).to(dev),
                                     torch.from_numpy(z["weights"]).to(dev))
    assert O.rel_l2(z["out"], y.cpu().numpy()) <= 1e-5
