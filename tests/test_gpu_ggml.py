"""The ggml op adapter (latent_ggml_pack_layer + latent_ggml_expert_ffn) through
the C ABI, the way ggml_cuda_latent_expert_ffn would call it
(kernels/latent_fused_expert_ffn.cu:134-292): raw row-major stacked factor
tensors as the reference GGUF writer stores them (loader/write_latent_gguf.py:
101-123) are repacked on the device, then the op runs with F16 x, F16 router
weights and the per-slot F32 dst, and with the combined dst.

Layers: the reference-written fixture tests/golden/latent_layer.gguf (B
factors of rank 13 padded to 32 here), and config 0's layer written in the
same layout (d 1024, f 704: the wide B factors go through the tile repack).
Oracle: per routed slot swiglu_expert on the reference's factors with the
same f16-rounded x; rel-L2 <= 1e-5.
"""

import ctypes as C
from dataclasses import replace

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN, golden
from gpu_helpers import decode, rel
from latent_b200 import _lib, synth

pytestmark = pytest.mark.gpu
TOL = 1e-5
ORDER = [("gate", "a"), ("gate", "b"), ("up", "a"), ("up", "b"), ("down", "a"), ("down", "b")]


def _gt(t: torch.Tensor, ne, typ):
    g = _lib.GgmlTensor()
    g.data = t.data_ptr()
    for i, v in enumerate(list(ne) + [1] * (4 - len(ne))):
        g.ne[i] = v
    g.type = typ
    return g


def _pack(raw, dev):
    """raw {(kind, side): (codes [E, rows, cols/2] uint8, scales [E, rows, cols/32] fp16)} -> (desc, buffers)."""
    keep, arr = [], (_lib.GgmlTensor * 12)()
    for i, key in enumerate(ORDER):
        codes, scales = raw[key]
        c = torch.from_numpy(np.ascontiguousarray(codes)).to(dev)
        s = torch.from_numpy(np.ascontiguousarray(scales).view(np.int16)).to(dev)
        keep += [c, s]
        arr[2 * i] = _gt(c, codes.shape, _lib.GGML_I8)
        arr[2 * i + 1] = _gt(s, scales.shape, _lib.GGML_F16)
    lib, stream = _lib.lib(), torch.cuda.current_stream().cuda_stream
    need = C.c_size_t()
    desc = _lib.FfnDesc()
    _lib.check(lib.latent_ggml_pack_layer(arr, None, 0, C.byref(need), None, stream), "size")
    buf = torch.empty(need.value, dtype=torch.uint8, device=dev)
    _lib.check(lib.latent_ggml_pack_layer(arr, buf.data_ptr(), buf.numel(), C.byref(need), C.byref(desc), stream),
               "pack")
    torch.cuda.synchronize()
    del keep                                   # the sources may go once the stream has passed the pack
    return desc, buf


def _run(desc, x, ids, w, per_slot):
    dev = x.device
    T, k = ids.shape
    d = desc.n_embd
    out = torch.full((T, k, d) if per_slot else (T, d), float("nan"), device=dev)
    src = (_lib.GgmlTensor * 3)(_gt(x, (d, T), _lib.GGML_F16), _gt(ids, (k, T), _lib.GGML_I32),
                                _gt(w, (k, T), _lib.GGML_F16))
    dst = _gt(out, (d, k, T) if per_slot else (d, T), _lib.GGML_F32)
    lib, stream = _lib.lib(), torch.cuda.current_stream().cuda_stream
    need = C.c_size_t()
    _lib.check(lib.latent_ggml_expert_ffn(C.byref(desc), src, C.byref(dst), None, 0, C.byref(need), stream), "ws")
    ws = torch.empty(max(need.value, 256), dtype=torch.uint8, device=dev)
    _lib.check(lib.latent_ggml_expert_ffn(C.byref(desc), src, C.byref(dst), ws.data_ptr(), ws.numel(), None,
                                          stream), "latent_ggml_expert_ffn")
    d2 = _lib.FfnDesc.from_buffer_copy(desc)
    d2.n_tokens, d2.top_k, d2.workspace, d2.workspace_bytes = T, k, ws.data_ptr(), ws.numel()
    _lib.check(lib.latent_expert_ffn_check(C.byref(d2), stream), "check")
    return out.cpu().numpy()


def _reference(x16, ids, w16, pairs, per_slot):
    x = x16.float().cpu().numpy()
    ids_np, w = ids.cpu().numpy(), w16.float().cpu().numpy()
    T, k = ids_np.shape
    if not per_slot:
        return O.moe_forward(x, ids_np, w, pairs)
    out = np.zeros((T, k, x.shape[1]), np.float64)
    for t in range(T):
        for j in range(k):
            e = int(ids_np[t, j])
            if e >= 0:
                out[t, j] = O.swiglu_expert(x[t:t + 1], *pairs[e])[0]
    return out


def _check_layer(raw, pairs, x, ids, w):
    dev = x.device
    desc, buf = _pack(raw, dev)
    for key, qm in zip(ORDER, (desc.gate_a, desc.gate_b, desc.up_a, desc.up_b, desc.down_a, desc.down_b)):
        for e in range(desc.n_expert):
            got = torch.empty((qm.rows, qm.cols), dtype=torch.float32, device=dev)
            _lib.check(_lib.lib().latent_dequantize(C.byref(qm), e, got.data_ptr(),
                                                    torch.cuda.current_stream().cuda_stream), "dequant")
            want = pairs[e][("gate", "up", "down").index(key[0])][0 if key[1] == "a" else 1]
            g = got.cpu().numpy()
            assert np.array_equal(g[:want.shape[0], :want.shape[1]].view(np.uint32), want.view(np.uint32)), key
            assert not g[want.shape[0]:].any() and not g[:, want.shape[1]:].any(), key
    for per_slot in (True, False):
        got = _run(desc, x, ids, w, per_slot)
        assert rel(_reference(x, ids, w, pairs, per_slot), got) <= TOL, per_slot


def test_reference_fixture_through_the_ggml_adapter(cuda):
    from latent_b200 import gguf_io
    pytest.importorskip("gguf")
    z = golden("gguf_layer")
    raw = gguf_io.read_layer(GOLDEN / "latent_layer.gguf", int(z["layer"]))
    def pad_b(a, b):                           # B rows (largest actual rank) padded to A's max_rank with zeros
        out = np.zeros((a.shape[1], b.shape[1]), np.float32)
        out[:b.shape[0]] = b
        return out
    pairs = [tuple((z[f"e{e}/{n}_a"], pad_b(z[f"e{e}/{n}_a"], z[f"e{e}/{n}_b"])) for n in ("gate", "up", "down"))
             for e in range(int(z["E"]))]
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(z["x"]).to(dev).half()
    ids = torch.from_numpy(z["ids"]).to(dev)
    w = torch.from_numpy(z["weights"]).to(dev).half()
    _check_layer(raw, pairs, x, ids, w)


def test_wide_layer_through_the_ggml_adapter(cuda):
    cfg = replace(synth.CONFIGS[0], snr_db=None)      # GGUF v0 carries NF4 groups only
    facs = synth.make_expert_factors(cfg, "cpu")
    raw = {}
    for kind, side in ORDER:
        fs = [ex[f"{kind}_{side}"] for ex in facs]
        rows, cols = fs[0].rows, fs[0].cols
        codes = np.stack([f.lo.numpy().reshape(rows, cols // 2) for f in fs])
        scales = np.stack([f.scales.numpy().view(np.float16).reshape(rows, cols // 32) for f in fs])
        raw[(kind, side)] = (codes, scales)
    pairs = [tuple((decode(ex[f"{n}_a"]), decode(ex[f"{n}_b"])) for n in ("gate", "up", "down")) for ex in facs]
    dev = torch.device("cuda", 0)
    x, ids, w = synth.make_batch(cfg, dev, n_tokens=24, seed_offset=5)
    ids[3, 1] = -1
    _check_layer(raw, pairs, x.half(), ids, w.half())
