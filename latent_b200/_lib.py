"""ctypes binding of the C ABI in ``include/latent_ffn.h``.

The structs below mirror the header field for field.  The library is loaded
from ``latent_b200/_lib/liblatent_b200.so`` (built in-tree by
``python -m latent_b200.build``); there is no fallback -- a missing or
unloadable library raises.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblatent_b200.so"

LATENT_OK = 0
STATUS_NAMES = {
    0: "LATENT_OK", 1: "LATENT_ERR_INVALID", 2: "LATENT_ERR_SHAPE", 3: "LATENT_ERR_DTYPE",
    4: "LATENT_ERR_ALIGN", 5: "LATENT_ERR_EXPERT_ID", 6: "LATENT_ERR_WORKSPACE",
    7: "LATENT_ERR_TIMEOUT", 8: "LATENT_ERR_CUDA", 9: "LATENT_ERR_UNSUPPORTED", 10: "LATENT_ERR_CAPACITY",
}

TYPE_F32, TYPE_F16, TYPE_BF16 = 0, 1, 2
FLAG_WEIGHT_BEFORE_DOWN = 1 << 0
FLAG_OUT_PER_SLOT = 1 << 1
ROUTER_RENORMALIZE = 1 << 0
ROUTER_SOFTMAX = 1 << 1
PATH_AUTO, PATH_DECODE, PATH_PREFILL = 0, 1, 2

# Every entry point the header declares, with (restype, argtypes).
EXPORTS = {}


class QMatrix(C.Structure):
    _fields_ = [
        ("codes", C.c_void_p),
        ("scales", C.c_void_p),
        ("i8_mask", C.c_void_p),
        ("i8_base", C.c_void_p),
        ("i8_hi", C.c_void_p),
        ("i8_blocks", C.c_void_p),
        ("i8_list", C.c_void_p),
        ("rows", C.c_int64),
        ("cols", C.c_int64),
    ]


class FfnDesc(C.Structure):
    _fields_ = [
        ("n_expert", C.c_int32),
        ("n_embd", C.c_int32),
        ("n_ff", C.c_int32),
        ("rank", C.c_int32),
        ("n_tokens", C.c_int32),
        ("top_k", C.c_int32),
        ("x_type", C.c_int32),
        ("w_type", C.c_int32),
        ("flags", C.c_uint32),
        ("path", C.c_int32),
        ("x", C.c_void_p),
        ("ids", C.c_void_p),
        ("weights", C.c_void_p),
        ("out", C.c_void_p),
        ("gate_a", QMatrix),
        ("gate_b", QMatrix),
        ("up_a", QMatrix),
        ("up_b", QMatrix),
        ("down_a", QMatrix),
        ("down_b", QMatrix),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
    ]


class DenseExpert(C.Structure):
    _fields_ = [
        ("expert", C.c_int32),
        ("rank", C.c_int32),
        ("dense", C.c_void_p * 3),
        ("a", C.c_void_p * 3),
        ("b", C.c_void_p * 3),
    ]


class DenseDesc(C.Structure):
    _fields_ = [
        ("n_expert", C.c_int32),
        ("n_embd", C.c_int32),
        ("n_ff", C.c_int32),
        ("n_tokens", C.c_int32),
        ("top_k", C.c_int32),
        ("x_type", C.c_int32),
        ("w_type", C.c_int32),
        ("dense_type", C.c_int32),
        ("flags", C.c_uint32),
        ("n_dense", C.c_int32),
        ("experts", C.POINTER(DenseExpert)),
        ("dense_index", C.c_void_p),
        ("x", C.c_void_p),
        ("ids", C.c_void_p),
        ("weights", C.c_void_p),
        ("out", C.c_void_p),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
    ]


class GgmlTensor(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("ne", C.c_int64 * 4),
        ("type", C.c_int32),
    ]


GGML_F32, GGML_F16, GGML_I8, GGML_I32, GGML_BF16 = 0, 1, 24, 26, 30


class EpDesc(C.Structure):
    _fields_ = [
        ("n_expert", C.c_int32),
        ("n_embd", C.c_int32),
        ("n_tokens", C.c_int32),
        ("top_k", C.c_int32),
        ("x_type", C.c_int32),
        ("w_type", C.c_int32),
        ("flags", C.c_uint32),
        ("x", C.c_void_p),
        ("ids", C.c_void_p),
        ("weights", C.c_void_p),
        ("send_x", C.c_void_p),
        ("send_expert", C.c_void_p),
        ("send_weight", C.c_void_p),
        ("expert_counts", C.c_void_p),
        ("y_back", C.c_void_p),
        ("out", C.c_void_p),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
    ]


EXPORTS.update({
    "latent_ep_workspace_size": (C.c_int, [C.POINTER(EpDesc), C.POINTER(C.c_size_t)]),
    "latent_ep_dispatch": (C.c_int, [C.POINTER(EpDesc), C.c_void_p]),
    "latent_ep_combine": (C.c_int, [C.POINTER(EpDesc), C.c_void_p]),
    "latent_ep_check": (C.c_int, [C.POINTER(EpDesc), C.c_void_p]),
    "latent_ep_pack_fixed_merged": (C.c_int, [C.POINTER(EpDesc), C.c_int32, C.c_int32, C.c_void_p, C.c_size_t,
                                              C.POINTER(C.c_size_t), C.c_void_p]),
    "latent_ep_unpack_fixed": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                         C.c_int32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p]),
    "latent_dense_workspace_size": (C.c_int, [C.POINTER(DenseDesc), C.POINTER(C.c_size_t)]),
    "latent_quantize_groups": (C.c_int, [C.c_void_p, C.c_int64, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_void_p]),
    "latent_ggml_pack_layer": (C.c_int, [C.POINTER(GgmlTensor), C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t),
                                         C.POINTER(FfnDesc), C.c_void_p]),
    "latent_ggml_expert_ffn": (C.c_int, [C.POINTER(FfnDesc), C.POINTER(GgmlTensor), C.POINTER(GgmlTensor),
                                         C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t), C.c_void_p]),
    "latent_dense_experts_prepare": (C.c_int, [C.POINTER(DenseDesc), C.c_void_p, C.c_void_p]),
    "latent_dense_experts_forward": (C.c_int, [C.POINTER(DenseDesc), C.c_void_p]),
    "latent_dense_matmul": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_int64,
                                      C.c_int64, C.c_int64, C.c_void_p]),
    "latent_abi_version": (C.c_int, []),
    "latent_status_string": (C.c_char_p, [C.c_int]),
    "latent_expert_ffn_workspace_size": (C.c_int, [C.POINTER(FfnDesc), C.POINTER(C.c_size_t)]),
    "latent_expert_ffn_forward": (C.c_int, [C.POINTER(FfnDesc), C.c_void_p]),
    "latent_expert_ffn_check": (C.c_int, [C.POINTER(FfnDesc), C.c_void_p]),
    "latent_expert_ffn_forward_noalloc": (C.c_int, [C.POINTER(FfnDesc), C.c_void_p]),
    "latent_expert_ffn_check_noalloc": (C.c_int, [C.POINTER(FfnDesc), C.c_void_p]),
    "latent_debug_set_wait_limit": (C.c_int, [C.c_uint64, C.c_int32]),
    "latent_expert_ffn_forward_timed": (C.c_int, [C.POINTER(FfnDesc), C.c_void_p, C.POINTER(C.c_void_p), C.c_int]),
    "latent_dequantize": (C.c_int, [C.POINTER(QMatrix), C.c_int32, C.c_void_p, C.c_void_p]),
    "latent_silu": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "latent_ep_pack_fixed": (C.c_int, [C.POINTER(EpDesc), C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "latent_ep_combine_fixed": (C.c_int, [C.POINTER(EpDesc), C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                          C.c_void_p]),
    "latent_router_topk": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_double, C.c_uint32,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "latent_router_route": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_double, C.c_uint32,
                                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "latent_pack_tiles": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
                                    C.c_void_p]),
})

_lock = threading.Lock()
_lib = None


class LatentError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{what}: {name}" if what else name)


def lib() -> C.CDLL:
    """The loaded CUDA library (raises if it is missing or stale)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m latent_b200.build` "
                    "(latent_b200 has no CPU fallback)")
            h = C.CDLL(str(LIB_PATH))
            for name, (res, args) in EXPORTS.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            if h.latent_abi_version() != 4:
                raise RuntimeError("liblatent_b200.so ABI version mismatch")
            _lib = h
    return _lib


def check(status: int, what: str = "") -> None:
    if status != LATENT_OK:
        raise LatentError(status, what)
