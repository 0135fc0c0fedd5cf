"""GPU: the load-time repack (latent_pack_tiles) matches the Python packer byte for byte."""
import numpy as np
import pytest
import torch

from latent_b200 import format as F
from latent_b200.runtime import pack_tiles


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(64, 704), (32, 256), (96, 1408), (40, 96)])
def test_pack_tiles_matches_host_order(cuda, rows, cols):
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(rows + cols)
    E = 3
    codes = torch.from_numpy(rng.integers(0, 256, (E, rows, cols // 2), dtype=np.uint8))
    sc = rng.integers(0, 0x7BFF, (E, rows, cols // 32)).astype(np.uint16)
    sc[rng.random(sc.shape) < 0.1] |= 0x8000  # INT8 flags pass through
    scales = torch.from_numpy(sc.view(np.int16))
    dc, ds = pack_tiles(codes.to(dev), scales.to(dev), rows, cols)
    perm = F.tile_order(rows, cols)
    want_c = codes.reshape(E, -1, 16)[:, perm]
    want_s = scales.reshape(E, -1)[:, perm]
    assert torch.equal(dc.cpu(), want_c)
    assert torch.equal(ds.cpu(), want_s)


@pytest.mark.gpu
def test_pack_tiles_rejects_bad_arguments(cuda):
    from latent_b200 import _lib
    c = torch.zeros((1, 32, 16), dtype=torch.uint8, device="cuda")
    s = torch.zeros((1, 32, 1), dtype=torch.int16, device="cuda")
    lib = _lib.lib()
    assert lib.latent_pack_tiles(c.data_ptr(), s.data_ptr(), 1, 32, 33, c.data_ptr(), s.data_ptr(), None) == 2
    assert lib.latent_pack_tiles(c.data_ptr(), s.data_ptr(), 1, 32, 32, c.data_ptr(), s.data_ptr(), None) == 1
