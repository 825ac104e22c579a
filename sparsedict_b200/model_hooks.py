"""Hooks that put SparseDict's model attention calls on this library's kernels.

The reference models build the dense ``(B, N, E*M)`` score tensor and call
``sparse_topk_attention`` on it; its ``use_fused_kernel=True`` switch
(``models/moe_topk_restorer.py:355-360``) was reserved for a fused kernel that
the reference never shipped.  These functions are the fused replacements of
the two call sites, with the same arguments:

* ``fused_mixture(module, query_tokens, branch, bank, top_k, gates=None)`` —
  ``DualDomainMoEDictionary._mixture`` (``models/modules/dual_domain_moe.py:139-174``);
  ``install_fused_mixture(module)`` binds it onto a module instance in place
  of the dense method.
* ``fused_token_attention(queries, keys, values, gates, top_k, tau)`` — the
  token-routed restorer's block (``models/moe_topk_restorer.py:162-172``):
  ``(q·k + log g)`` with ``-inf`` where ``g == 0``, divided by
  ``tau * sqrt(d_k)``, top-k attention over the flat atoms.

Both return the attention output ``(B, N, C)`` and are differentiable in the
queries, the atom projections and the gates, as the dense path is.
"""

from __future__ import annotations

import math
import types

import torch

from .mixture import gated_mixture_attention


def fused_mixture(module, query_tokens: torch.Tensor, branch: int, bank: torch.Tensor, top_k: int,
                  gates: torch.Tensor | None = None) -> torch.Tensor:
    """``_mixture`` of a ``DualDomainMoEDictionary``-like ``module`` on the fused kernels.

    Uses the module's own projections: ``module.projections[branch]["query"]``
    for the queries and ``module._atom_projections(branch, bank)`` for the
    ``(E, M, d_k)`` keys and ``(E, M, C)`` values.
    """
    proj = module.projections[branch]
    q = proj["query"](query_tokens)
    keys, values = module._atom_projections(branch, bank)
    if gates is not None:
        gates = gates.to(q.dtype).contiguous()
    return gated_mixture_attention(q.contiguous(), keys.contiguous(), values.contiguous(), top_k, gates)


def install_fused_mixture(module):
    """Replace ``module._mixture`` (this instance only) by ``fused_mixture``; returns ``module``."""
    module._mixture = types.MethodType(fused_mixture, module)
    return module


def fused_token_attention(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                          gates: torch.Tensor | None, top_k: int, tau: float) -> torch.Tensor:
    """Gate-folded, temperature-scaled top-k attention of queries ``(B, N, d_k)``
    over expert atoms ``keys (E, M, d_k)`` / ``values (E, M, C)``."""
    if not isinstance(tau, (int, float)) or isinstance(tau, bool) or not tau > 0:
        raise ValueError(f"tau must be a positive number; got {tau}")
    scale = 1.0 / (float(tau) * math.sqrt(queries.shape[-1]))
    if gates is not None:
        gates = gates.to(queries.dtype).contiguous()
    return gated_mixture_attention(queries.contiguous(), keys.contiguous(), values.contiguous(), top_k, gates,
                                   scale=scale)
