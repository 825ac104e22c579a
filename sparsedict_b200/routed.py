"""Routed dictionary attention: the top-1 expert MoE use of the top-k op.

SparseDict's ``DualDomainMoEDictionary._mixture``
(``models/modules/dual_domain_moe.py:139-174``) scores every token against
all ``E*M`` atoms, folds the router gates in as ``+log(g)`` with ``-inf``
for disabled experts, and runs the dense top-k attention over the flat atom
axis.  With top-1 routing (``models/modules/router.py:139-145``) the gate of
the chosen expert is exactly 1 and every other expert is masked, so the
operation is: token ``n`` attends, with top-k selection, to the atoms of
expert ``argmax(logits[n])`` only, the atoms serving as both keys and values.

Here that runs without the dense ``(N, E*M)`` score tensor: a routing kernel
groups tokens by expert (stable counting sort), the fused forward treats
each expert as one slice of a ragged batch (reading queries through the
routing permutation), and the backward writes the key and value gradients of
an expert's dictionary into one buffer (``dDict = dK + dV``).
"""

from __future__ import annotations

import torch

from . import _native, _ops


class RoutedDictionaryAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, queries, dictionaries, router_logits, k, scale):
        logits = router_logits.detach().float().contiguous()
        expert, order, offsets = _ops.route_top1(logits)
        out, idx, lse, _ = _ops.topk_attn_fwd(
            queries, dictionaries, dictionaries, k, scale, row_offsets=offsets, row_index=order
        )
        ctx.save_for_backward(queries, dictionaries, idx, lse, order, offsets)
        ctx.scale = scale
        ctx.mark_non_differentiable(expert)
        return out, expert, idx

    @staticmethod
    def backward(ctx, grad_out, _g_expert, _g_idx):
        queries, dictionaries, idx, lse, order, offsets = ctx.saved_tensors
        # keys and values are one dictionary: one gradient buffer receives dK + dV
        dq, ddict, _ = _ops.topk_attn_bwd_out(
            queries, dictionaries, dictionaries, grad_out.to(queries.dtype).contiguous(), idx, lse, ctx.scale,
            row_offsets=offsets, row_index=order, shared_kv=True,
        )
        return dq, ddict, None, None, None


def routed_dictionary_attention(
    queries: torch.Tensor,
    dictionaries: torch.Tensor,
    router_logits: torch.Tensor,
    k: int,
    scale: float = 1.0,
    return_routing: bool = False,
):
    """Top-k attention of each token within its top-1 expert's dictionary.

    ``queries`` ``(N, d)``, ``dictionaries`` ``(E, M, d)`` (keys = values),
    ``router_logits`` ``(N, E)``.  ``scale`` multiplies the raw dot products;
    ``_mixture`` applies none (1.0).  Returns ``(N, d)``; with
    ``return_routing`` also the int32 expert per token and the selected atom
    indices (local to the expert, in expert-grouped row order).
    """
    if queries.ndim != 2 or dictionaries.ndim != 3 or router_logits.ndim != 2:
        raise ValueError("expected queries (N, d), dictionaries (E, M, d) and router_logits (N, E)")
    n, d = queries.shape
    e, m, dd = dictionaries.shape
    if dd != d:
        raise ValueError(f"query/atom feature sizes must match; got {d} and {dd}")
    if tuple(router_logits.shape) != (n, e):
        raise ValueError(f"expected router_logits of shape {(n, e)}; got {tuple(router_logits.shape)}")
    if not isinstance(k, int) or isinstance(k, bool) or not 1 <= k <= m:
        raise ValueError(f"k must be an integer in [1, {m}]; got {k}")
    if queries.dtype != dictionaries.dtype:
        raise ValueError("queries and dictionaries must share one dtype")
    if not (queries.is_contiguous() and dictionaries.is_contiguous()):
        raise ValueError("queries and dictionaries must be contiguous")
    if queries.device.type != "cuda" or dictionaries.device != queries.device or router_logits.device != queries.device:
        raise ValueError("routed path requires CUDA tensors on one device")
    if not _native.available():
        raise RuntimeError("the sparsedict_b200 native library is required; build it with "
                           "`python -m sparsedict_b200.build`")
    out, expert, idx = RoutedDictionaryAttention.apply(queries, dictionaries, router_logits, k, float(scale))
    return (out, expert, idx) if return_routing else out
