"""B200-native fused latent expert FFN (LATENT's GGML_OP_LATENT_EXPERT_FFN path).

Public API mirrors the reference CPU runtime (loader/latent_runtime.py) plus
the batched routed op:

    from latent_b200 import load_pair, swiglu_expert, moe_expert_ffn, ExpertSet
"""

from .format import ExpertSet, GroupedFactor, StackedFactor, from_int8, from_mixed, from_nf4, from_npz
from .quant import quantize_factor
from .runtime import (ExpertFFN, FactorPair, dense_swiglu_expert, dequantize, load_pair, moe_expert_ffn,
                      project, router_topk, silu, swiglu_expert, workspace_bytes)

__all__ = [
    "ExpertSet", "GroupedFactor", "StackedFactor", "from_int8", "from_mixed", "from_nf4", "from_npz",
    "quantize_factor", "ExpertFFN", "FactorPair", "dense_swiglu_expert", "dequantize", "load_pair",
    "moe_expert_ffn", "project", "router_topk", "silu", "swiglu_expert", "workspace_bytes",
]
