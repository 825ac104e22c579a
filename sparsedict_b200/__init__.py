"""sparsedict_b200: SparseDict's fused top-k sparse attention, native to B200 (sm_100a).

Public API (the reference's names and signatures):
    fused_topk_attention, FusedTopKAttentionFunction, hybrid_topk_attention,
    tiled_affinity, tiled_topk, tiled_topk_aggregate
plus per-query adaptive k (``adaptive_topk_attention``), routed dictionary
attention (``routed_dictionary_attention``), the gated
mixture over a bank of dictionary atoms (``gated_mixture_attention``, the
``_mixture`` of SparseDict's MoE dictionary, with the model hooks of
``sparsedict_b200.model_hooks``) and the row-sharded multi-GPU step
(``sparsedict_b200.sharded``); the selection operators of SparseDict's
``topk_select`` module over given scores live in ``sparsedict_b200.selection``.
"""

from .kernels.fused_topk_attn import (
    FusedTopKAttentionFunction,
    fused_topk_attention,
    tiled_affinity,
    tiled_topk,
    tiled_topk_aggregate,
)
from .kernels.hybrid_topk import _hybrid_topk_attention_with_aux, hybrid_topk_attention
from ._ops import deterministic_backward, set_deterministic_backward
from .adaptive import AdaptiveTopKAttentionFunction, adaptive_topk_attention
from .mixture import GatedMixtureFunction, gated_mixture_attention
from .model_hooks import fused_mixture, fused_token_attention, install_fused_mixture
from .routed import RoutedDictionaryAttention, routed_dictionary_attention
from .sharded import ShardedTopKAttention, ShardPlan

__all__ = [
    "AdaptiveTopKAttentionFunction",
    "adaptive_topk_attention",
    "FusedTopKAttentionFunction",
    "ShardPlan",
    "ShardedTopKAttention",
    "deterministic_backward",
    "set_deterministic_backward",
    "GatedMixtureFunction",
    "gated_mixture_attention",
    "fused_mixture",
    "fused_token_attention",
    "install_fused_mixture",
    "RoutedDictionaryAttention",
    "routed_dictionary_attention",
    "fused_topk_attention",
    "hybrid_topk_attention",
    "tiled_affinity",
    "tiled_topk",
    "tiled_topk_aggregate",
]
