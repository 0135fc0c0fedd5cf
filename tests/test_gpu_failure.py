"""Failure paths of the decode kernel, made without a GPU fault.

The fused decode kernel bounds every device-side wait; a wait that runs out
records LATENT_ERR_TIMEOUT in the workspace and the kernel unwinds (its bulk
copies land before the CTAs exit).  The test hook latent_debug_set_wait_limit
shortens the limit to 20 ms and makes each cross-CTA dependency wait ask for
one completion more than any CTA will make -- a flag that nothing sets -- so
the wait runs out on purpose.  The host must then read the timeout through
latent_expert_ffn_check, and the context must stay usable: the next call,
with the defaults restored, is correct and reports no error.
"""

import pytest
import torch

from conftest import golden
from gpu_helpers import golden_moe_experts, rel
from latent_b200 import ExpertFFN, ExpertSet, _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def layer(cuda):
    z = golden("moe")
    facs, _ = golden_moe_experts(z)
    es = ExpertSet(facs, device="cuda")
    x = torch.from_numpy(z["x"]).cuda()
    ids = torch.from_numpy(z["ids"]).cuda()
    w = torch.from_numpy(z["weights"]).cuda()
    return ExpertFFN(es, path="decode"), x, ids, w


def test_unreachable_dependency_times_out_and_the_context_survives(layer):
    op, x, ids, w = layer
    lib = _lib.lib()
    ref = op(x, ids, w).clone()
    op.check()
    assert lib.latent_debug_set_wait_limit(20_000_000, 1) == 0
    try:
        op(x, ids, w)
        with pytest.raises(_lib.LatentError) as info:
            op.check()
        assert info.value.status == 7          # LATENT_ERR_TIMEOUT
    finally:
        assert lib.latent_debug_set_wait_limit(0, 0) == 0
    y = op(x, ids, w)
    op.check()
    assert torch.isfinite(y).all()
    assert rel(ref.cpu().numpy(), y) <= 1e-6


def test_short_wait_limit_alone_does_not_time_out(layer):
    op, x, ids, w = layer
    lib = _lib.lib()
    ref = op(x, ids, w).clone()
    assert lib.latent_debug_set_wait_limit(20_000_000, 0) == 0
    try:
        for _ in range(3):
            y = op(x, ids, w)
            op.check()
    finally:
        assert lib.latent_debug_set_wait_limit(0, 0) == 0
    assert rel(ref.cpu().numpy(), y) <= 1e-6

