"""The C-ABI library loads without a GPU, exports every declared entry point,
and rejects bad descriptors on the host before touching the device."""

import ctypes as C
import re
from pathlib import Path

import pytest

from latent_b200 import _lib
from latent_b200.build import build

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    text = (ROOT / "include" / "latent_ffn.h").read_text()
    return set(re.findall(r"LATENT_API\s+[\w\s\*]+?\b(latent_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.lib()


def test_exports_match_header(lib):
    declared = _declared()
    assert {"latent_expert_ffn_forward", "latent_expert_ffn_workspace_size", "latent_dequantize"} <= declared
    assert declared == set(_lib.EXPORTS), "ctypes binding and header disagree"
    for name in declared:
        assert hasattr(lib, name), name


def test_wait_limit_hook_validates_on_the_host(lib):
    assert lib.latent_debug_set_wait_limit(10, 0) == 1             # below 1 ms
    assert lib.latent_debug_set_wait_limit(10 ** 12, 0) == 1       # above the 2 s default
    assert lib.latent_debug_set_wait_limit(50_000_000, 1) == 0
    assert lib.latent_debug_set_wait_limit(0, 0) == 0               # defaults back


def test_version_and_status_strings(lib):
    assert lib.latent_abi_version() == 4
    assert lib.latent_status_string(0) == b"ok"
    assert b"expert id" in lib.latent_status_string(5)


def _desc(E=4, d=64, f=96, r=32, T=3, k=2):
    dsc = _lib.FfnDesc()
    dsc.n_expert, dsc.n_embd, dsc.n_ff, dsc.rank, dsc.n_tokens, dsc.top_k = E, d, f, r, T, k
    for kind, (rows, cols) in {"gate_a": (d, r), "up_a": (d, r), "down_a": (f, r),
                               "gate_b": (r, f), "up_b": (r, f), "down_b": (r, d)}.items():
        q = getattr(dsc, kind)
        q.rows, q.cols = rows, cols
    return dsc


def test_workspace_size_and_validation(lib):
    dsc = _desc()
    n = C.c_size_t()
    assert lib.latent_expert_ffn_workspace_size(C.byref(dsc), C.byref(n)) == 0
    assert n.value > 0 and n.value % 256 == 0
    empty = _desc(T=0)         # empty batch: valid, small workspace
    assert lib.latent_expert_ffn_workspace_size(C.byref(empty), C.byref(n)) == 0
    bad = _desc(d=48)          # not a multiple of 32
    assert lib.latent_expert_ffn_workspace_size(C.byref(bad), C.byref(n)) == 2
    bad = _desc(r=96)          # unsupported padded rank
    assert lib.latent_expert_ffn_workspace_size(C.byref(bad), C.byref(n)) == 9
    bad = _desc()
    bad.gate_b.cols = 64       # inconsistent factor shape
    assert lib.latent_expert_ffn_workspace_size(C.byref(bad), C.byref(n)) == 2
    bad = _desc()
    bad.x_type = 7
    assert lib.latent_expert_ffn_workspace_size(C.byref(bad), C.byref(n)) == 3
    assert lib.latent_expert_ffn_workspace_size(None, C.byref(n)) == 1


def test_forward_rejects_null_pointers_on_host(lib):
    dsc = _desc()
    assert lib.latent_expert_ffn_forward(C.byref(dsc), None) == 1  # LATENT_ERR_INVALID, nothing launched
    dsc0 = _desc(T=0)
    assert lib.latent_expert_ffn_forward(C.byref(dsc0), None) == 0  # empty batch is a no-op


def test_dequantize_and_silu_validate_on_host(lib):
    q = _lib.QMatrix()
    assert lib.latent_dequantize(C.byref(q), 0, None, None) == 1
    assert lib.latent_silu(None, None, -1, None) == 1
    assert lib.latent_silu(None, None, 0, None) == 0


def test_router_topk_validates_on_host(lib):
    f = lib.latent_router_topk
    assert f(None, 4, 8, 9, 0.9, 0, None, None, None, None) == 2        # top_k > n_expert
    assert f(None, 4, 8, 0, 0.9, 0, None, None, None, None) == 2        # top_k < 1
    assert f(None, 4, 8, 2, 0.0, 0, None, None, None, None) == 1        # threshold outside (0, 1]
    assert f(None, 4, 8, 2, 1.5, 0, None, None, None, None) == 1
    assert f(None, 4, 8, 2, 0.9, 4, None, None, None, None) == 1        # unknown flag
    assert f(None, 4, 2048, 2, 0.9, 0, None, None, None, None) == 9     # beyond 1024 experts
    assert f(None, 4, 64, 33, 0.9, 0, None, None, None, None) == 9      # beyond top_k 32
    assert f(None, 0, 8, 2, 0.9, 0, None, None, None, None) == 0        # empty batch: nothing to do
    assert f(None, 4, 8, 2, 0.9, 0, None, None, None, None) == 1        # missing buffers
