"""Adaptive top-k router on the GPU (latent_router_topk) against the
reference's adaptive_topk_batch (loader/adaptive_topk.py:59-90, recorded in
tests/golden/router.npz) and the oracle restatement.

Integer outputs (ids, kept counts) are bit-exact; the renormalised weights
are float32 divisions of the same operands on both sides, so they are
compared bit for bit too."""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden
from latent_b200 import router_topk

pytestmark = pytest.mark.gpu


def _run(scores, k, th, renorm=True):
    ids, w, nk = router_topk(torch.from_numpy(scores).cuda(), k, th, renormalize=renorm)
    return ids.cpu().numpy(), w.cpu().numpy(), nk.cpu().numpy()


def test_router_matches_reference_golden(cuda):
    z = golden("router")
    for c in range(int(z["n_cases"])):
        scores, k, th = z[f"c{c}/scores"], int(z[f"c{c}/top_k"]), float(z[f"c{c}/threshold"])
        ids, w, nk = _run(scores, k, th)
        keep = z[f"c{c}/keep"]
        assert np.array_equal(nk, z[f"c{c}/n_kept"]), c
        assert np.array_equal(ids >= 0, keep), c
        assert np.array_equal(ids[keep], z[f"c{c}/order"][keep]), c
        _, w_ref, _ = O.router_topk(scores, k, th)
        assert np.array_equal(w.view(np.uint32), w_ref.view(np.uint32)), c


@pytest.mark.parametrize("T,E,k,th", [(16384, 256, 8, 0.95), (333, 1024, 32, 0.9), (77, 1000, 6, 0.5),
                                      (50, 1, 1, 1.0), (64, 64, 6, 1.0), (129, 33, 7, 0.7)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_matches_oracle(cuda, T, E, k, th, renorm):
    rng = np.random.default_rng(T + E + k)
    logits = rng.standard_normal((T, E)) * 2.0
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    scores = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
    ids, w, nk = _run(scores, k, th, renorm)
    ids_o, w_o, nk_o = O.router_topk(scores, k, th, renormalize=renorm)
    assert np.array_equal(nk, nk_o)
    assert np.array_equal(ids, ids_o)
    assert np.array_equal(w.view(np.uint32), w_o.view(np.uint32))


def test_router_ties_zero_rows_and_empty(cuda):
    rng = np.random.default_rng(5)
    scores = (rng.integers(0, 4, size=(200, 48)) / 8.0).astype(np.float32)   # many equal scores
    scores[3] = 0.0
    ids, w, nk = _run(scores, 6, 0.8)
    ids_o, w_o, nk_o = O.router_topk(scores, 6, 0.8)
    assert np.array_equal(ids, ids_o) and np.array_equal(nk, nk_o)
    assert np.array_equal(w.view(np.uint32), w_o.view(np.uint32))
    assert nk[3] == 0 and (ids[3] == -1).all()
    ids, w, nk = router_topk(torch.empty((0, 16), device="cuda"), 2)
    assert ids.shape == (0, 2) and nk.shape == (0,)


def test_router_nan_rows_follow_numpy_sort_order(cuda):
    """numpy's argsort places NaN after every number: a NaN is picked only
    when fewer than k numbers remain, and then the NaN total keeps all k
    slots with NaN weights."""
    rng = np.random.default_rng(6)
    scores = rng.random((6, 48)).astype(np.float32)
    scores[1, 7] = np.nan                         # one NaN, k numbers left: never picked
    scores[2, 3:] = np.nan                        # 3 numbers, then NaN in expert order
    scores[3, :] = np.nan                         # all NaN
    scores[4, ::2] = np.nan
    for renorm in (True, False):
        ids, w, nk = _run(scores, 6, 0.8, renorm)
        ids_o, w_o, nk_o = O.router_topk(scores, 6, 0.8, renormalize=renorm)
        assert np.array_equal(ids, ids_o) and np.array_equal(nk, nk_o)
        assert np.array_equal(np.isnan(w), np.isnan(w_o))
        fin = ~np.isnan(w_o)
        assert np.array_equal(w[fin].view(np.uint32), w_o[fin].view(np.uint32))
        assert sorted(ids[2][:3]) == [0, 1, 2] and list(ids[2][3:]) == [3, 4, 5] and nk[2] == 6
        assert np.isnan(w[2]).all() == renorm
        assert 7 not in ids[1]
    ids, w, nk = router_topk(torch.empty((0, 16), device="cuda"), 2)
    assert ids.shape == (0, 2) and nk.shape == (0,)


def test_router_feeds_the_fused_op(cuda):
    """Router output straight into the fused op equals the oracle MoE on the same routing."""
    from latent_b200 import ExpertFFN, ExpertSet
    from latent_b200 import format as F
    z = golden("moe")
    facs, pairs = [], []
    for e in range(int(z["E"])):
        arrays = {kk.split("/", 1)[1]: z[kk] for kk in z.files if kk.startswith(f"e{e}/")}
        facs.append({f"{n}_{s}": F.from_npz(arrays, n, s) for n in ("gate", "up", "down") for s in ("a", "b")})
        pairs.append(tuple(O.pair_from_npz(arrays, n) for n in ("gate", "up", "down")))
    E = int(z["E"])
    x = z["x"]
    rng = np.random.default_rng(9)
    logits = rng.standard_normal((x.shape[0], E))
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    scores = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
    ids, w, _ = router_topk(torch.from_numpy(scores).cuda(), 2, 0.6)
    y = ExpertFFN(ExpertSet(facs, device=torch.device("cuda", 0)), path="decode")(torch.from_numpy(x).cuda(), ids, w)
    ids_o, w_o, _ = O.router_topk(scores, 2, 0.6)
    ref = O.moe_forward(x, ids_o, w_o, pairs)
    assert O.rel_l2(ref, y.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("T,E,k,th", [(4096, 256, 8, 0.95), (333, 64, 6, 0.8), (50, 1024, 32, 0.9)])
def test_fused_softmax_router_and_histogram(cuda, T, E, k, th):
    """latent_router_route with logits: the softmax (fp32, max-subtracted) runs
    in the selection kernel.  Against the oracle on numpy's float32 softmax of
    the same logits: ids and kept counts equal wherever no two of a token's
    probabilities (or a running sum and the threshold target) are within
    1e-5 relative of each other; weights within 1e-6; the per-expert counts
    equal the histogram of the kept ids."""
    rng = np.random.default_rng(T + E)
    logits = (rng.standard_normal((T, E)) * 2.0).astype(np.float32)
    ids, w, nk, counts = router_topk(torch.from_numpy(logits).cuda(), k, th, logits=True, expert_counts=True)
    ids, w, nk, counts = ids.cpu().numpy(), w.cpu().numpy(), nk.cpu().numpy(), counts.cpu().numpy()
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    p = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
    ids_o, w_o, nk_o = O.router_topk(p, k, th)
    top = -np.sort(-p, axis=1)[:, :k + 1]
    close = (np.abs(np.diff(top, axis=1)) <= 1e-5 * top[:, 1:]).any(axis=1)
    tot = top[:, :k].sum(axis=1, dtype=np.float32)
    cum = np.cumsum(top[:, :k], axis=1)
    close |= (np.abs(cum - th * tot[:, None]) <= 1e-5 * tot[:, None]).any(axis=1)
    ok = ~close
    assert ok.mean() > 0.9
    assert np.array_equal(ids[ok], ids_o[ok]) and np.array_equal(nk[ok], nk_o[ok])
    assert np.allclose(w[ok], w_o[ok], rtol=1e-6, atol=1e-7)
    want = np.bincount(ids[ids >= 0].ravel(), minlength=E)
    assert np.array_equal(counts, want)
    # probabilities in, through the same entry point: bit-exact with latent_router_topk
    ids2, w2, nk2 = router_topk(torch.from_numpy(p).cuda(), k, th)
    ids3, w3, nk3 = O.router_topk(p, k, th)
    assert np.array_equal(ids2.cpu().numpy(), ids3) and np.array_equal(nk2.cpu().numpy(), nk3)

