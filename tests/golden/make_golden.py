"""Generate the golden vectors that pin the CPU oracle to the reference.

Run once, from the repository root, with a checkout of the reference
(Yxmura/latent) available:

    python tests/golden/make_golden.py --reference <path-to-latent-checkout>

The script imports the reference's own ``loader/latent_loader.py`` and
``loader/latent_runtime.py``, feeds them seeded inputs and records inputs and
outputs as small ``.npz`` fixtures next to this file.  The fixtures are
committed; nothing at test or bench time needs the reference checkout.

Fixtures:
  nf4.npz      quantize_nf4 / dequantize_nf4 cases (odd counts, zero groups, g16/g32)
  int8.npz     quantize_int8 / dequantize_int8 cases (g64 and g32)
  mixed.npz    per-group NF4 -> INT8 fallback built from the reference's
               encoders and SNR applied group by group
  runtime.npz  compress_matrix artifacts (reference NPZ keys) + swiglu_expert
               outputs, NF4 and whole-pair INT8, with/without weight_before_down
  latent_layer.gguf + gguf_layer.npz
               one MoE layer stacked by the reference's compress_layer_to_stacked
               (loader/write_latent_gguf.py:126-275) and written with its tensor
               names and byte layout (:412-436); the npz holds the reference
               dequantized factors of every expert and a routed batch with the
               reference swiglu_expert outputs combined in fp64
  router.npz   adaptive_topk_batch (loader/adaptive_topk.py) on softmax router
               scores: keep masks, kept counts and the reference's top-k order
               for several (E, k, threshold), an all-zero row, k = E
  moe.npz      a small routed MoE layer: per-expert artifacts, x, ids (with -1
               slots), weights, per-slot outputs of the reference swiglu_expert
               and the fp64 top-k combine
  compress.npz the reference compressor's stages on two spectral matrices:
               full singular values, choose_rank, the seeded Gaussian test
               matrix, randomized_svd + make_factors (float A, B),
               quantize_nf4 bytes of A and B, compress_matrix's report
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _ref_modules(ref_root: Path):
    sys.path.insert(0, str(ref_root))
    from loader import latent_loader as ll  # noqa: E402
    from loader import latent_runtime as lr  # noqa: E402
    return ll, lr


def _compress(ll, name, matrix, rank, seed, force_int8=False):
    arrays, report = ll.compress_matrix(
        name=name, matrix=matrix, energy=0.999999, min_rank=rank, max_rank=rank,
        group_size=32, int8_group_size=64, error_threshold=10.0,
        snr_threshold=1e9 if force_int8 else 0.0,
        low_snr_fraction_threshold=0.0 if force_int8 else 1.0, seed=seed)
    assert not report.fallback
    return arrays, report


def _spectral(rng, m, n, r):
    """W = U diag(s) V^T (+1e-4 noise) with Haar U, V and s_i = 0.5 i^-0.8."""
    k = min(m, n)
    qu, ru = np.linalg.qr(rng.standard_normal((m, k)))
    qv, rv = np.linalg.qr(rng.standard_normal((n, k)))
    qu *= np.sign(np.diag(ru))
    qv *= np.sign(np.diag(rv))
    s = 0.5 * np.arange(1, k + 1, dtype=np.float64) ** -0.8
    w = (qu * s) @ qv.T + 1e-4 * rng.standard_normal((m, n))
    return w.astype(np.float32)


def make_nf4(ll):
    rng = np.random.default_rng(11)
    cases = [
        (np.linspace(-2.0, 2.0, 133, dtype=np.float32).reshape(7, 19), 16),
        (rng.standard_normal((64, 96)).astype(np.float32), 32),
        (rng.standard_normal(33).astype(np.float32), 32),
        (np.concatenate([np.zeros(32, np.float32), rng.standard_normal(32).astype(np.float32) * 1e-3]), 32),
        ((rng.standard_normal((5, 64)) * np.logspace(-4, 3, 64)).astype(np.float32), 32),
        # exact midpoints between levels exercise the argmin tie rule
        (np.concatenate([[1.0], (ll.NF4_CODEBOOK[:-1] + ll.NF4_CODEBOOK[1:]) / 2,
                         np.zeros(16)]).astype(np.float32), 32),
    ]
    out = {}
    for i, (v, g) in enumerate(cases):
        packed, scales, shape = ll.quantize_nf4(v, group_size=g)
        out[f"c{i}.values"] = v
        out[f"c{i}.group"] = np.int32(g)
        out[f"c{i}.packed"] = packed
        out[f"c{i}.scales"] = scales
        out[f"c{i}.shape"] = np.array(shape, np.int64)
        out[f"c{i}.decoded"] = ll.dequantize_nf4(packed, scales, shape, group_size=g)
    out["n_cases"] = np.int32(len(cases))
    np.savez_compressed(HERE / "nf4.npz", **out)


def make_int8(ll):
    rng = np.random.default_rng(12)
    cases = [
        (rng.standard_normal((64, 96)).astype(np.float32), 64),
        (rng.standard_normal(33).astype(np.float32), 64),
        (rng.standard_normal((16, 32)).astype(np.float32) * 50, 32),
        (np.concatenate([np.zeros(64, np.float32), np.full(64, 0.5, np.float32)]), 64),
    ]
    out = {}
    for i, (v, g) in enumerate(cases):
        q, scales, shape = ll.quantize_int8(v, group_size=g)
        out[f"c{i}.values"] = v
        out[f"c{i}.group"] = np.int32(g)
        out[f"c{i}.q"] = q
        out[f"c{i}.scales"] = scales
        out[f"c{i}.shape"] = np.array(shape, np.int64)
        out[f"c{i}.decoded"] = ll.dequantize_int8(q, scales, shape, group_size=g)
    out["n_cases"] = np.int32(len(cases))
    np.savez_compressed(HERE / "int8.npz", **out)


def make_mixed(ll):
    rng = np.random.default_rng(13)
    v = rng.standard_normal((16, 64)).astype(np.float32)
    v[:, 5] *= 40.0   # outlier column: its groups lose SNR under NF4
    v[3, :] *= 1e-3
    g = 32
    flat = v.reshape(-1, g)
    nf4_packed, scales, is_i8, q_all, decoded = [], [], [], [], []
    for row in flat:
        p, s, sh = ll.quantize_nf4(row, group_size=g)
        dq = ll.dequantize_nf4(p, s, sh, group_size=g)
        snr = ll.quantization_snr_by_group(row, dq, g)[0]
        nf4_packed.append(p)
        if snr < np.float32(10.0):
            q, s8, sh8 = ll.quantize_int8(row, group_size=g)
            scales.append(s8[0])
            is_i8.append(True)
            q_all.append(q)
            decoded.append(ll.dequantize_int8(q, s8, sh8, group_size=g))
        else:
            scales.append(s[0])
            is_i8.append(False)
            q_all.append(np.zeros(g, np.int8))
            decoded.append(dq)
    np.savez_compressed(
        HERE / "mixed.npz", values=v, nf4=np.concatenate(nf4_packed),
        scales=np.array(scales, np.float16), is_int8=np.array(is_i8),
        int8=np.concatenate(q_all), decoded=np.concatenate(decoded).reshape(v.shape))


def make_compress(ll):
    rng = np.random.default_rng(31)
    out = {}
    cases = [(256, 192, 0.9, 8, 64, 5), (192, 320, 0.999, 64, 64, 9)]   # (m, n, energy, min, max, seed)
    for i, (m, n, energy, rmin, rmax, seed) in enumerate(cases):
        w = _spectral(rng, m, n, 0)
        full_s = np.linalg.svd(w, compute_uv=False)
        rank = ll.choose_rank(full_s, energy=energy, min_rank=rmin, max_rank=rmax)
        u, s, vt = ll.randomized_svd(w, target_rank=rank, seed=seed)
        a, b = ll.make_factors(u, s, vt, rank)
        ap, asc, _ = ll.quantize_nf4(a, group_size=32)
        bp, bsc, _ = ll.quantize_nf4(b, group_size=32)
        _, report = ll.compress_matrix(
            name="w", matrix=w, energy=energy, min_rank=rmin, max_rank=rmax, group_size=32, int8_group_size=64,
            error_threshold=10.0, snr_threshold=0.0, low_snr_fraction_threshold=1.0, seed=seed)
        out.update({f"c{i}.w": w, f"c{i}.energy": np.float64(energy), f"c{i}.min_rank": np.int32(rmin),
                    f"c{i}.max_rank": np.int32(rmax), f"c{i}.seed": np.int32(seed), f"c{i}.full_s": full_s,
                    f"c{i}.rank": np.int32(rank), f"c{i}.a": a, f"c{i}.b": b, f"c{i}.a_nf4": ap,
                    f"c{i}.a_scales": asc, f"c{i}.b_nf4": bp, f"c{i}.b_scales": bsc,
                    f"c{i}.dense_error": np.float64(report.dense_relative_error),
                    f"c{i}.quant_error": np.float64(report.quantized_relative_error),
                    f"c{i}.retained": np.float64(report.retained_energy)})
    out["n_cases"] = np.int32(len(cases))
    np.savez_compressed(HERE / "compress.npz", **out)


def make_runtime(ll, lr):
    rng = np.random.default_rng(14)
    d, f, r = 64, 96, 32
    out = {}
    mats = {"gate": _spectral(rng, d, f, 48), "up": _spectral(rng, d, f, 48), "down": _spectral(rng, f, d, 48)}
    for variant, force in (("nf4", False), ("int8", True)):
        arrays = {}
        for i, (name, m) in enumerate(mats.items()):
            a, rep = _compress(ll, name, m, r, seed=20 + i, force_int8=force)
            assert rep.quantization.startswith(variant), rep.quantization
            arrays.update(a)
        for k, val in arrays.items():
            out[f"{variant}/{k}"] = val
        x = rng.standard_normal((5, d)).astype(np.float32)
        gate, up, down = (lr.load_pair(arrays, n) for n in ("gate", "up", "down"))
        out[f"{variant}/x"] = x
        out[f"{variant}/y"] = lr.swiglu_expert(x, gate, up, down)
        out[f"{variant}/y_wbd"] = lr.swiglu_expert(x, gate, up, down, weight=0.3, weight_before_down=True)
        out[f"{variant}/dense_y"] = lr.dense_swiglu_expert(x, mats["gate"], mats["up"], mats["down"])
    for k, m in mats.items():
        out[f"dense/{k}"] = m
    np.savez_compressed(HERE / "runtime.npz", **out)


def make_moe(ll, lr):
    rng = np.random.default_rng(15)
    E, d, f, r, T, k = 4, 64, 96, 32, 12, 2
    out = {"E": np.int32(E), "k": np.int32(k)}
    pairs = []
    for e in range(E):
        arrays = {}
        for i, (name, (m, n)) in enumerate((("gate", (d, f)), ("up", (d, f)), ("down", (f, d)))):
            a, _ = _compress(ll, name, _spectral(rng, m, n, 48), r, seed=100 + 3 * e + i)
            arrays.update(a)
        for key, val in arrays.items():
            out[f"e{e}/{key}"] = val
        pairs.append(tuple(lr.load_pair(arrays, n) for n in ("gate", "up", "down")))
    x = rng.standard_normal((T, d)).astype(np.float32)
    logits = rng.standard_normal((T, E))
    ids = np.argsort(-logits, axis=1)[:, :k].astype(np.int32)
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    w = np.take_along_axis(p, ids, axis=1)
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    ids[2, 1] = -1          # skipped slots contribute nothing
    ids[7, 0] = -1
    per_slot = np.zeros((T, k, d), np.float32)
    per_slot_wbd = np.zeros((T, k, d), np.float32)
    for t in range(T):
        for j in range(k):
            e = ids[t, j]
            if e < 0:
                continue
            g, u, dn = pairs[e]
            per_slot[t, j] = lr.swiglu_expert(x[t:t + 1], g, u, dn)[0]
            per_slot_wbd[t, j] = lr.swiglu_expert(x[t:t + 1], g, u, dn, weight=float(w[t, j]),
                                                  weight_before_down=True)[0]
    live = (ids >= 0)[:, :, None]
    out.update(x=x, ids=ids, weights=w, per_slot=per_slot, per_slot_wbd=per_slot_wbd,
               out=(per_slot.astype(np.float64) * w[:, :, None] * live).sum(axis=1).astype(np.float32),
               out_wbd=(per_slot_wbd.astype(np.float64) * live).sum(axis=1).astype(np.float32))
    np.savez_compressed(HERE / "moe.npz", **out)


def make_router(ref_root: Path):
    from loader import adaptive_topk as at  # noqa: E402
    rng = np.random.default_rng(11)
    out = {}
    cases = [(8, 2, 0.95), (64, 6, 0.95), (64, 6, 0.5), (256, 8, 0.95), (256, 8, 1.0), (16, 16, 0.9),
             (40, 12, 0.8)]
    for c, (E, k, th) in enumerate(cases):
        logits = rng.standard_normal((96, E)) * (1.0 + c % 3)
        p = np.exp(logits - logits.max(axis=1, keepdims=True))
        scores = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
        scores[5] = 0.0                                   # total <= 0: nothing kept
        keep, n_kept = at.adaptive_topk_batch(scores, k, th)
        order = np.argsort(-scores, axis=1)[:, :k].astype(np.int32)
        out.update({f"c{c}/scores": scores, f"c{c}/top_k": np.int32(k), f"c{c}/threshold": np.float64(th),
                    f"c{c}/keep": keep, f"c{c}/n_kept": n_kept, f"c{c}/order": order})
    out["n_cases"] = np.int32(len(cases))
    np.savez_compressed(HERE / "router.npz", **out)


def make_gguf(ll, lr, ref_root: Path):
    import gguf
    from loader import write_latent_gguf as wl  # noqa: E402
    rng = np.random.default_rng(21)
    E, d, f, layer = 3, 64, 96, 5
    # numpy write order of the GGUF reader: (n_out, n_in, n_expert)
    gate = np.stack([_spectral(rng, d, f, 32).T for _ in range(E)], axis=2).astype(np.float32)
    up = np.stack([_spectral(rng, d, f, 32).T for _ in range(E)], axis=2).astype(np.float32)
    down = np.stack([_spectral(rng, f, d, 32).T for _ in range(E)], axis=2).astype(np.float32)
    wt, st, reports, ranks = wl.compress_layer_to_stacked(
        layer_idx=layer, gate_exps=gate, up_exps=up, down_exps=down, energy=0.9, min_rank=8, max_rank=32,
        group_size=32, int8_group_size=64, error_threshold=10.0, snr_threshold=0.0,
        low_snr_fraction_threshold=1.0)
    w = gguf.GGUFWriter(str(HERE / "latent_layer.gguf"), arch="deepseek4", use_temp_file=False)
    for name, arr in wt.items():           # same byte layout as write_latent_gguf.py:426-431
        w.add_tensor(name, arr.astype(np.int8).reshape(arr.shape[2], arr.shape[1], arr.shape[0]),
                     raw_dtype=gguf.GGMLQuantizationType.I8)
    for name, arr in st.items():
        w.add_tensor(name, arr.astype(np.float16).reshape(arr.shape[2], arr.shape[1], arr.shape[0]),
                     raw_dtype=gguf.GGMLQuantizationType.F16)
    w.add_tensor(f"blk.{layer}.ffn_latent_ranks", ranks.T.astype(np.uint8), raw_dtype=gguf.GGMLQuantizationType.I8)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    out = {"E": np.int32(E), "layer": np.int32(layer), "ranks": ranks}
    dense = {}
    for kind in ("gate", "up", "down"):
        for ab in ("a", "b"):
            codes, scales = wt[f"blk.{layer}.ffn_latent_{kind}_{ab}"], st[f"blk.{layer}.ffn_latent_{kind}_{ab}_s"]
            n_e, rows, half = codes.shape
            for e in range(E):
                vals = np.stack([ll.dequantize_nf4(codes[e, i], scales[e, i], (2 * half,), group_size=32)
                                 for i in range(rows)])
                dense[(e, kind, ab)] = vals.astype(np.float32)
                out[f"e{e}/{kind}_{ab}"] = dense[(e, kind, ab)]
    T, k = 12, 2
    x = rng.standard_normal((T, d)).astype(np.float32)
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    ids[1, 1] = -1
    wts = rng.random((T, k)).astype(np.float32)
    res = np.zeros((T, d), np.float64)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            if e < 0:
                continue
            pr = []
            for kind in ("gate", "up", "down"):
                a, b = dense[(e, kind, "a")], dense[(e, kind, "b")]
                r = min(a.shape[1], b.shape[0])     # B rows = the largest actual rank; A cols = max_rank
                pr.append(lr.FactorPair(a[:, :r], b[:r]))
            y = lr.swiglu_expert(x[t:t + 1], *pr)
            res[t] += float(wts[t, j]) * y[0].astype(np.float64)
    out.update(x=x, ids=ids, weights=wts, out=res.astype(np.float32))
    np.savez_compressed(HERE / "gguf_layer.npz", **out)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path, help="checkout of Yxmura/latent")
    args = ap.parse_args()
    ll, lr = _ref_modules(args.reference)
    make_nf4(ll)
    make_int8(ll)
    make_mixed(ll)
    make_compress(ll)
    make_runtime(ll, lr)
    make_moe(ll, lr)
    make_router(args.reference)
    make_gguf(ll, lr, args.reference)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
