"""Host-side packing and quantization against the oracle (CPU only)."""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden
from latent_b200 import format as F
from latent_b200.quant import quantize_factor


def _decode(gf: F.GroupedFactor) -> np.ndarray:
    return O.decode_grouped(gf.lo.cpu().numpy(), gf.hi.cpu().numpy(), gf.scales.cpu().numpy().view(np.uint16),
                            gf.is_int8.cpu().numpy(), gf.rows, gf.cols)


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("variant", ["nf4", "int8"])
def test_reference_npz_factors_decode_bit_exact(variant):
    z = golden("runtime")
    arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(variant + "/")}
    for name in ("gate", "up", "down"):
        for side in ("a", "b"):
            gf = F.from_npz(arrays, name, side)
            ref = O.factor_from_npz(arrays, name, side)
            assert np.array_equal(_bits(_decode(gf)), _bits(ref)), (variant, name, side)
            assert bool(gf.is_int8.all()) == (variant == "int8")


def test_mixed_golden_decodes_bit_exact():
    z = golden("mixed")
    gf = F.from_mixed(z["nf4"], z["scales"], z["is_int8"], z["int8"], z["values"].shape)
    assert np.array_equal(_bits(_decode(gf)), _bits(z["decoded"]))


def test_missing_factor_raises_keyerror():
    z = golden("runtime")
    arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith("nf4/") and not k.endswith(".nf4")}
    with pytest.raises(KeyError):
        F.from_npz(arrays, "gate", "a")


def test_unaligned_columns_rejected():
    packed, scales, shape = O.nf4_encode(np.ones((4, 12), np.float32))
    with pytest.raises(ValueError):
        F.from_nf4(packed, scales, shape)


@pytest.mark.parametrize("snr_db", [None, 20.0, 35.0])
def test_quantizer_matches_oracle_encoders(snr_db):
    rng = np.random.default_rng(3)
    v = rng.standard_normal((48, 96)).astype(np.float32)
    v[:, 7] *= 30.0            # outlier column -> low-SNR groups
    v[5] = 0.0                 # all-zero groups
    v[6, :30] = O.NF4_LEVELS[:-1].tolist() + O.NF4_LEVELS[1:].tolist()  # exact levels in a group
    v[6, 31] = 1.0
    gf = quantize_factor(torch.from_numpy(v), snr_db)
    if snr_db is None:
        packed, scales, _ = O.nf4_encode(v)
        assert np.array_equal(gf.lo.numpy().ravel(), packed)
        assert np.array_equal(gf.scales.numpy().ravel().view(np.uint16), scales.view(np.uint16))
        assert not gf.is_int8.any()
    else:
        enc = O.mixed_encode(v, snr_db=snr_db)
        assert np.array_equal(gf.is_int8.numpy().ravel(), enc["is_int8"])
        assert enc["is_int8"].any()
        assert np.array_equal(gf.scales.numpy().ravel().view(np.uint16), enc["scales"].view(np.uint16))
        assert np.array_equal(_bits(_decode(gf)), _bits(O.mixed_decode(enc)))


def test_quantizer_tie_midpoints_pick_lowest_code():
    lv = O.NF4_LEVELS
    mids = ((lv[:-1] + lv[1:]) / 2).astype(np.float32)
    v = np.zeros((1, 32), np.float32)
    v[0, 0] = 1.0
    v[0, 1:16] = mids
    packed, _, _ = O.nf4_encode(v)
    gf = quantize_factor(torch.from_numpy(v), None)
    assert np.array_equal(gf.lo.numpy().ravel(), packed)


def test_padding_and_stacking_roundtrip():
    rng = np.random.default_rng(4)
    fs = []
    for e in range(3):
        v = rng.standard_normal((40, 64)).astype(np.float32)
        v[:, 3] *= 50
        fs.append(quantize_factor(torch.from_numpy(v), 20.0))
    padded = [f.padded(40, 128) for f in fs]
    for f, p in zip(fs, padded):
        dp = _decode(p)
        assert np.array_equal(_bits(dp[:, :64]), _bits(_decode(f)))
        assert not dp[:, 64:].any()
    st = F.StackedFactor(padded, "cpu")
    assert st.n_int8 == sum(f.n_int8 for f in fs) > 0
    for e, p in enumerate(padded):
        back = st.expert(e)
        assert np.array_equal(_bits(_decode(back)), _bits(_decode(p)))
    # the mask/base tables describe the compact sidecar
    m = st.i8_mask.numpy().view(np.uint32)
    base = st.i8_base.numpy()
    counts = np.array([[bin(int(w)).count("1") for w in row] for row in m])
    assert np.array_equal(base.ravel(), np.concatenate([[0], np.cumsum(counts.ravel())[:-1]]))


def test_expert_set_pads_rank_and_counts_bytes():
    rng = np.random.default_rng(5)
    d, f, r = 64, 96, 32
    ex = {}
    for name, (m, n) in (("gate", (d, f)), ("up", (d, f)), ("down", (f, d))):
        ex[f"{name}_a"] = quantize_factor(torch.from_numpy(rng.standard_normal((m, r)).astype(np.float32)), None)
        ex[f"{name}_b"] = quantize_factor(torch.from_numpy(rng.standard_normal((r, n)).astype(np.float32)), None)
    es = F.ExpertSet([ex, ex], device="cpu", rank=64)
    assert es.rank == 64 and es["gate_a"].cols == 64 and es["down_b"].rows == 64
    per = 3 * (d * 64 + 64 * f) + 3 * 0  # elements per expert... 3 A (rows*64) + 3 B (64*cols)
    elems = 2 * d * 64 + f * 64 + 2 * 64 * f + 64 * d
    assert es.factor_bytes([0]) == elems // 2 + elems // 32 * 2


def test_tile_major_order_of_wide_factors():
    """Factors wider than 256 columns are stored in 256-column tile-major group order."""
    rng = np.random.default_rng(6)
    rows, cols = 40, 704  # tiles of 256, 256 and 192 columns
    fs = []
    for e in range(2):
        v = rng.standard_normal((rows, cols)).astype(np.float32)
        v[:, 5] *= 60  # some INT8 groups
        fs.append(quantize_factor(torch.from_numpy(v), 20.0))
    st = F.StackedFactor(fs, "cpu")
    assert st.n_int8 > 0
    perm = F.tile_order(rows, cols).numpy()
    gpr = cols // 32
    assert perm.shape == (rows * gpr,) and sorted(perm.tolist()) == list(range(rows * gpr))
    # flat position q of (row, col): tile c, then row, then group within the tile
    for row, col in ((0, 0), (3, 40), (7, 300), (39, 703), (12, 512)):
        c = col // 256
        ng = min(8, gpr - 8 * c)
        q = c * rows * 8 + row * ng + (col - 256 * c) // 32
        assert perm[q] == row * gpr + col // 32
    for e, f in enumerate(fs):
        lo = f.lo.reshape(-1, 16).numpy()
        assert np.array_equal(st.codes[e].numpy(), lo[perm])
        sc = f.scales.reshape(-1).numpy().view(np.uint16)
        i8 = f.is_int8.reshape(-1).numpy()
        want = np.where(i8[perm], sc[perm] | 0x8000, sc[perm])
        assert np.array_equal(st.scales[e].numpy().view(np.uint16), want)
        back = st.expert(e)
        assert np.array_equal(_bits(_decode(back)), _bits(_decode(f)))
    # INT8 records follow the flat order of each expert
    m = st.i8_mask.numpy().view(np.uint32)
    bits = ((m[:, :, None].astype(np.uint64) >> np.arange(32, dtype=np.uint64)) & 1).reshape(2, -1)[:, : rows * gpr]
    first = 0
    for e, f in enumerate(fs):
        hi = f.hi.reshape(-1, 16).numpy()[perm]
        sel = bits[e].astype(bool)
        n = int(sel.sum())
        assert np.array_equal(st.i8_hi[first:first + n].numpy(), hi[sel])
        first += n


@pytest.mark.parametrize("rows,cols", [(352, 96), (64, 512), (256, 288)])
def test_int8_block_lists_match_brute_force(rows, cols):
    """Every INT8 group appears once in its (expert, tile, 128-row block) list,
    under its column, in row order, with its record index in (expert, q) order."""
    rng = np.random.default_rng(rows + cols)
    E, g = 3, rows * cols // 32
    is_i8 = torch.from_numpy(rng.random((E, g)) < 0.07)
    is_i8[1] = False                                     # an expert without INT8 groups
    words, entries = F.int8_block_lists(is_i8, rows, cols)
    words, entries = words.numpy().astype(np.int64), entries.numpy().astype(np.int64)
    tiles, rblk = (cols + 255) // 256, (rows + F.BLOCK_ROWS - 1) // F.BLOCK_ROWS
    assert words.shape == (E * tiles * rblk, F.BLOCK_WORDS)
    want = {}
    rec = 0
    for e in range(E):
        for q in range(g):
            c, within = divmod(q, rows * 8)
            ng = min(cols // 32 - 8 * c, 8)
            row, gi = divmod(within, ng)
            if is_i8[e, q]:
                want.setdefault((e * tiles + c) * rblk + row // F.BLOCK_ROWS, []).append((gi, row % F.BLOCK_ROWS, rec))
                rec += 1
    seen = 0
    for b in range(words.shape[0]):
        w = words[b]
        got = want.get(b, [])
        assert w[0] == 0 and w[8] == len(got) and w[9] % 4 == 0
        if not got:
            continue
        assert w[10] == min(r for _, _, r in got)
        for j in range(8):
            col = sorted((row, r) for gi, row, r in got if gi == j)
            ent = entries[w[9] + w[j]: w[9] + w[j + 1]]
            assert [(int(v) >> 16, (int(v) & 0xFFFF) + w[10]) for v in ent] == col, (b, j)
        seen += len(got)
    assert seen == int(is_i8.sum())


def test_int8_metadata_bytes_follow_the_block_lists():
    """nbytes counts what the decode kernel stages for INT8: 48 bytes of block
    words plus the padded entries of every block holding INT8 groups."""
    rng = np.random.default_rng(8)
    fs = []
    for e in range(3):
        v = rng.standard_normal((160, 288)).astype(np.float32)
        v[:, 5 + e] *= 60.0
        fs.append(quantize_factor(torch.from_numpy(v), 20.0))
    st = F.StackedFactor(fs, "cpu")
    assert st.n_int8 > 0
    words = st.i8_blocks.numpy().astype(np.int64)
    per_block = np.where(words[:, 8] > 0, 48 + (words[:, 8] + 3) // 4 * 16, 0).reshape(3, -1)
    base = 160 * 288 // 2 + 160 * 288 // 32 * 2
    for e in range(3):
        assert st.nbytes([e]) == base + int(per_block[e].sum())
    assert st.nbytes() == 3 * base + int(per_block.sum())
