"""LATENT GGUF stacked-factor reader (latent_b200.gguf_io) against the
reference writer's layout (loader/write_latent_gguf.py:126-275, 412-436).

tests/golden/latent_layer.gguf was written with the reference's stacking and
tensor records; gguf_layer.npz holds the reference's dequantized factors of
every expert and a routed batch with reference outputs."""

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN, golden
from latent_b200 import gguf_io

pytest.importorskip("gguf")


def test_reader_layout_matches_reference_dequant():
    z = golden("gguf_layer")
    raw = gguf_io.read_layer(GOLDEN / "latent_layer.gguf", int(z["layer"]))
    for (kind, side), (codes, scales) in raw.items():
        assert codes.shape[0] == int(z["E"])
        for e in range(int(z["E"])):
            want = z[f"e{e}/{kind}_{side}"]
            got = np.stack([O.nf4_decode(codes[e, i], scales[e, i], (codes.shape[2] * 2,))
                            for i in range(codes.shape[1])])
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (kind, side, e)


def test_missing_layer_raises_key_error():
    with pytest.raises(KeyError):
        gguf_io.read_layer(GOLDEN / "latent_layer.gguf", 0)
