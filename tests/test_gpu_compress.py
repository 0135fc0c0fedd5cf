"""GPU load-time compression (latent_b200.compress, kernel latent_quantize_groups).

Quantiser: byte-exact with the reference encoders -- the NF4 cases of
tests/golden/nf4.npz and the per-group NF4/INT8 cases of mixed.npz, both
made by the reference's own quantize_nf4 / quantize_int8
(loader/latent_loader.py:111-158) -- and with the torch restatement
(latent_b200.quant) on larger random factors with outlier columns.

Compressor: against the reference's compress_matrix stages recorded in
tests/golden/compress.npz (loader/latent_loader.py:66-108, 195-230): the
same rank, the same seeded test matrix, factors whose product matches the
reference's A.B to fp32 rounding (the SVD runs in cuSOLVER, not LAPACK), the
reference's dense error, and, for a rank that fills whole groups,
quantisation of the reference's own float factors byte-exact with its
quantize_nf4 bytes.  The compressed pair then runs through the routed op.
"""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden
from latent_b200 import compress, quant
from latent_b200.runtime import dequantize

pytestmark = pytest.mark.gpu


def _gpu_groups(values, snr_db):
    gf, snr = compress.quantize_groups(torch.from_numpy(np.ascontiguousarray(values, np.float32)).cuda(), snr_db)
    return gf, snr


def test_nf4_golden_cases_byte_exact(cuda):
    z = golden("nf4")
    n = 0
    for i in range(int(z["n_cases"])):
        v, g = z[f"c{i}.values"], int(z[f"c{i}.group"])
        if g != 32 or v.size % 32:
            continue
        gf, _ = _gpu_groups(v.reshape(-1, 32), None)
        assert np.array_equal(gf.lo.cpu().numpy().reshape(-1), z[f"c{i}.packed"]), i
        assert np.array_equal(gf.scales.cpu().numpy().view(np.float16).reshape(-1), z[f"c{i}.scales"]), i
        n += 1
    assert n >= 1


def test_mixed_golden_byte_exact(cuda):
    z = golden("mixed")
    gf, _ = _gpu_groups(z["values"], 20.0)
    i8 = gf.is_int8.cpu().numpy().reshape(-1)
    assert np.array_equal(i8, z["is_int8"])
    assert np.array_equal(gf.scales.cpu().numpy().view(np.float16).reshape(-1), z["scales"])
    lo = gf.lo.cpu().numpy().reshape(-1, 16)
    hi = gf.hi.cpu().numpy().reshape(-1, 16)
    nf4 = z["nf4"].reshape(-1, 16)
    assert np.array_equal(lo[~i8], nf4[~i8])
    q = z["int8"].reshape(-1, 32).view(np.uint8)
    want_lo = (q[:, 0::2] & 15) | ((q[:, 1::2] & 15) << 4)
    want_hi = (q[:, 0::2] >> 4) | ((q[:, 1::2] >> 4) << 4)
    assert np.array_equal(lo[i8], want_lo[i8]) and np.array_equal(hi[i8], want_hi[i8])
    assert np.array_equal(dequantize(gf).cpu().numpy().view(np.uint32), z["decoded"].view(np.uint32))


@pytest.mark.parametrize("snr_db", [None, 20.0, 30.0])
def test_kernel_matches_torch_restatement(cuda, snr_db):
    rng = np.random.default_rng(4)
    v = rng.standard_normal((384, 256)).astype(np.float32)
    v[:, 17] *= 60.0                     # outlier column
    v[5] = 0.0                           # all-zero groups stay NF4
    v[9, :64] *= 1e-30                   # tiny magnitudes
    ref = quant.quantize_factor(torch.from_numpy(v), snr_db)
    gf, snr = _gpu_groups(v, snr_db)
    if snr_db is not None:
        # groups within 1e-5 of the threshold may round differently (the norms' summation order): none here
        thr = 10.0 ** (snr_db / 20.0)
        assert not (abs(snr.cpu().numpy() / thr - 1.0) < 1e-5).any()
        assert gf.is_int8.any()
    for name in ("lo", "hi", "scales", "is_int8"):
        assert torch.equal(getattr(gf, name).cpu(), getattr(ref, name).cpu()), name


def test_compress_matrix_matches_reference_stages(cuda):
    z = golden("compress")
    for i in range(int(z["n_cases"])):
        w = z[f"c{i}.w"]
        res = compress.compress_matrix(w, energy=float(z[f"c{i}.energy"]), min_rank=int(z[f"c{i}.min_rank"]),
                                       max_rank=int(z[f"c{i}.max_rank"]), snr_db=None, error_threshold=10.0,
                                       seed=int(z[f"c{i}.seed"]))
        assert res.rank == int(z[f"c{i}.rank"]), i
        a, b = z[f"c{i}.a"], z[f"c{i}.b"]
        r = res.rank
        # the float product agrees with the reference's (SVD factors may differ in sign, not the product);
        # the quantised one is as far from W as the reference's
        ours = (res.a_float @ res.b_float).cpu().numpy()
        assert O.rel_l2(a @ b, ours) <= 1e-3
        assert abs(res.report["dense_relative_error"] - float(z[f"c{i}.dense_error"])) <= 1e-4
        q_ref = float(z[f"c{i}.quant_error"])
        assert abs(res.report["quantized_relative_error"] - q_ref) <= 0.05 * q_ref
        if r % 32 == 0:   # whole row groups: the reference's flat groups are the same groups
            gfa, _ = _gpu_groups(a, None)
            gfb, _ = _gpu_groups(b, None)
            assert np.array_equal(gfa.lo.cpu().numpy().reshape(-1), z[f"c{i}.a_nf4"])
            assert np.array_equal(gfb.lo.cpu().numpy().reshape(-1), z[f"c{i}.b_nf4"])
            assert np.array_equal(gfa.scales.cpu().numpy().view(np.float16).reshape(-1), z[f"c{i}.a_scales"])
            assert np.array_equal(gfb.scales.cpu().numpy().view(np.float16).reshape(-1), z[f"c{i}.b_scales"])


def test_compressed_expert_runs_in_the_routed_op(cuda):
    from latent_b200 import ExpertFFN, ExpertSet
    from gpu_helpers import decode
    rng = np.random.default_rng(12)
    d, f = 256, 352
    experts = []
    for e in range(3):
        ex = {}
        for name, (m, n) in (("gate", (d, f)), ("up", (d, f)), ("down", (f, d))):
            w = (rng.standard_normal((m, 48)) @ rng.standard_normal((48, n)) / 30.0).astype(np.float32)
            c = compress.compress_matrix(w, energy=0.999, min_rank=8, max_rank=64, snr_db=20.0, seed=e)
            ex[f"{name}_a"], ex[f"{name}_b"] = c.a, c.b
        experts.append(ex)
    es = ExpertSet([{k: v for k, v in ex.items()} for ex in experts], device="cuda")
    x = torch.from_numpy(rng.standard_normal((6, d)).astype(np.float32)).cuda()
    ids = torch.tensor([[0, 1], [2, 0], [1, 2], [0, -1], [2, 1], [1, 0]], dtype=torch.int32).cuda()
    wts = torch.full((6, 2), 0.5).cuda()
    y = ExpertFFN(es, path="decode")(x, ids, wts)
    table = []
    for ex in experts:
        table.append(tuple((decode(ex[f"{n}_a"].to("cpu")), decode(ex[f"{n}_b"].to("cpu")))
                           for n in ("gate", "up", "down")))
    ref = O.moe_forward(x.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy(), table)
    assert O.rel_l2(ref, y.cpu().numpy()) <= 1e-5

