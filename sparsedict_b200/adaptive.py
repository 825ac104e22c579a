"""Top-k attention with a per-query number of selected keys (adaptive k).

SparseDict's restorer predicts a per-token budget ``k_i`` and collapses it to
one integer before selection (``models/moe_topk_restorer.py:333-338``,
``_effective_top_k``; per-token k is listed future work,
``observations.md:63-65``).  Here every query keeps its own ``k_i``: row
``(b, h, n)`` is top-``k_i`` attention — the softmax over its ``k_i`` best
keys (larger score first, lower index on ties) and their values.  One fused
forward serves all rows with ``k_max = max k_i``: the selection bound is
computed for ``k_max`` (which bounds every smaller k), and each row's cut
keeps its own ``k_i``; the index slots past ``k_i`` hold -1, which the
backward skips.
"""

from __future__ import annotations

import math

import torch

from . import _native, _ops
from .kernels.fused_topk_attn import validate_fused_inputs


class AdaptiveTopKAttentionFunction(torch.autograd.Function):
    """Forward as ``FusedTopKAttentionFunction`` with a per-row k; saves the
    flattened inputs, the int32 indices (-1 past each row's k) and the LSE."""

    @staticmethod
    def forward(ctx, queries, keys, values, row_k, k_max, temperature=1.0):
        b, h, n, dq = queries.shape
        m, dv = keys.shape[2], values.shape[3]
        bh = b * h
        scale = 1.0 / (temperature * math.sqrt(dq))
        q2 = queries.reshape(bh, n, dq)
        k2 = keys.reshape(bh, m, dq)
        v2 = values.reshape(bh, m, dv)
        rk = row_k.reshape(bh * n).to(device=queries.device, dtype=torch.int32).contiguous()
        out, idx, lse, _ = _ops.topk_attn_fwd(q2, k2, v2, k_max, scale, row_k=rk)
        idx = idx.view(bh, n, k_max)
        lse = lse.view(bh, n)
        ctx.save_for_backward(q2, k2, v2, idx, lse)
        ctx.geometry = (b, h, n, dq, m, dv, scale)
        return out.view(b, h, n, dv)

    @staticmethod
    def backward(ctx, grad_output):
        q2, k2, v2, idx, lse = ctx.saved_tensors
        b, h, n, dq, m, dv, scale = ctx.geometry
        dout = grad_output.reshape(b * h, n, dv).to(q2.dtype).contiguous()
        dqg, dkg, dvg = _ops.topk_attn_bwd_out(q2, k2, v2, dout, idx, lse, scale)
        return (dqg.view(b, h, n, dq), dkg.view(b, h, m, dq), dvg.view(b, h, m, dv), None, None, None)


def adaptive_topk_attention(
    queries: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    k_per_query: torch.Tensor,
    temperature: float = 1.0,
    k_max: int | None = None,
) -> torch.Tensor:
    """Top-k attention where query ``(b, h, n)`` keeps ``k_per_query[b, h, n]`` keys.

    ``queries (B, H, N, D)``, ``keys (B, H, M, D)``, ``values (B, H, M, Dv)`` as
    ``fused_topk_attention``; ``k_per_query`` an integer tensor ``(B, H, N)``
    with values in ``[1, k_max]``.  ``k_max`` defaults to the tensor's maximum
    (read back to the host once).  Returns ``(B, H, N, Dv)``; differentiable in
    queries, keys and values.
    """
    if not isinstance(k_per_query, torch.Tensor):
        raise TypeError("k_per_query must be a torch.Tensor")
    if k_per_query.dtype not in (torch.int8, torch.int16, torch.int32, torch.int64, torch.uint8):
        raise ValueError(f"k_per_query must have an integer dtype; got {k_per_query.dtype}")
    if queries.ndim == 4 and tuple(k_per_query.shape) != tuple(queries.shape[:3]):
        raise ValueError(f"k_per_query must have shape {tuple(queries.shape[:3])}; got {tuple(k_per_query.shape)}")
    if k_per_query.numel() == 0:
        raise ValueError("k_per_query must be non-empty")
    lo, hi = (int(x) for x in torch.aminmax(k_per_query.to(torch.int64)))
    if k_max is None:
        k_max = hi
    if lo < 1 or hi > k_max:
        raise ValueError(f"k_per_query values must lie in [1, {k_max}]; got [{lo}, {hi}]")
    validate_fused_inputs(queries, keys, values, k_max, temperature)
    if k_per_query.device != queries.device:
        raise ValueError("k_per_query must be on the queries' device")
    _native.load()
    return AdaptiveTopKAttentionFunction.apply(queries, keys, values, k_per_query, int(k_max), float(temperature))
