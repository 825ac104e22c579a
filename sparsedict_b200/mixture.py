"""Gated top-k mixture over a bank of projected dictionary atoms.

SparseDict's ``DualDomainMoEDictionary._mixture``
(``models/modules/dual_domain_moe.py:139-174``) scores every token against
the atoms of all experts (``E*M`` of them, no score scale), folds the gates
in as ``+log(max(g, tiny))`` with ``-inf`` where a gate is 0, and runs top-k
attention over the flat atom axis (``models/modules/topk_select.py:106-162``).

Here that runs in the fused kernels without the dense ``(B, N, E*M)`` score
tensor: the gate fold is an additive score bias per (token, expert) applied
inside the selection (``sdk_topk_attn_fwd_biased``), and the backward returns
the bias gradient (the per-expert sum of dS over a token's selected atoms),
from which the gate gradient ``dS_sum / g`` follows, as autograd through the
reference's ``clamp_min(tiny).log()`` gives.  Without gates the op is plain
top-k attention over the flat atoms with scale 1.
"""

from __future__ import annotations

import torch

from . import _native, _ops


def _gate_bias(gates: torch.Tensor, rows: int, experts: int, acc: torch.dtype, tiny: float,
               scale: float = 1.0) -> torch.Tensor:
    g = gates.reshape(rows, experts).to(acc)
    bias = g.clamp_min(tiny).log() * scale
    return torch.where(g == 0, torch.full_like(bias, float("-inf")), bias).contiguous()


class GatedMixtureFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, queries, keys, values, gates, k, scale=1.0):
        b, n, dk = queries.shape
        e, m, _ = keys.shape
        c = values.shape[-1]
        rows = b * n
        acc = _ops.acc_dtype(queries.dtype)
        q2 = queries.reshape(1, rows, dk)
        k2 = keys.reshape(1, e * m, dk)
        v2 = values.reshape(1, e * m, c)
        tiny = torch.finfo(queries.dtype).tiny
        bias = None if gates is None else _gate_bias(gates, rows, e, acc, tiny, scale)
        out, idx, lse, _ = _ops.topk_attn_fwd(q2, k2, v2, k, scale, seg_bias=bias)
        ctx.save_for_backward(q2, k2, v2, idx, lse, gates, bias)
        ctx.shape = (b, n, dk, e, m, c)
        ctx.tiny = tiny
        ctx.scale = scale
        return out.reshape(b, n, c)

    @staticmethod
    def backward(ctx, grad_out):
        q2, k2, v2, idx, lse, gates, bias = ctx.saved_tensors
        b, n, dk, e, m, c = ctx.shape
        rows = b * n
        dout = grad_out.reshape(1, rows, c).to(q2.dtype).contiguous()
        dbias = None
        if bias is not None and ctx.needs_input_grad[3]:
            dbias = torch.empty((rows, e), device=q2.device, dtype=bias.dtype)
        dq, dk_acc, dv_acc = _ops.topk_attn_bwd(q2, k2, v2, dout, idx, lse, ctx.scale, seg_bias=bias,
                                                dseg_bias=dbias)
        dgates = None
        if dbias is not None:
            g = gates.reshape(rows, e).to(dbias.dtype)
            live = g >= ctx.tiny  # clamp_min passes the gradient; 0 gates are masked
            dgates = torch.where(live, dbias * ctx.scale / torch.where(live, g, torch.ones_like(g)),
                                 torch.zeros_like(g))
            dgates = dgates.reshape(b, n, e).to(gates.dtype)
        dkeys = _ops.finalize_grad(dk_acc, k2.dtype).reshape(e, m, dk)
        dvalues = _ops.finalize_grad(dv_acc, v2.dtype).reshape(e, m, c)
        return dq.reshape(b, n, dk), dkeys, dvalues, dgates, None, None


def gated_mixture_attention(
    queries: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    top_k: int,
    gates: torch.Tensor | None = None,
    scale: float = 1.0,
) -> torch.Tensor:
    """Softmax top-k mixture of each token over the projected atoms of all experts.

    ``queries`` ``(B, N, d_k)``, ``keys`` ``(E, M, d_k)``, ``values``
    ``(E, M, C)`` (the atom projections of ``_mixture``), optional ``gates``
    ``(B, N, E)``: a zero gate disables that expert for the token and nonzero
    gates are folded in additively (``+log g``), so the slots selected by the
    top-k come out renormalised together.  ``scale`` multiplies the folded
    score, ``(q·k + log g) * scale`` (SparseDict's token-routed restorer
    divides by ``tau * sqrt(d_k)`` after the fold, moe_topk_restorer.py:165-170);
    ``_mixture`` itself uses 1.  Returns ``(B, N, C)``; differentiable in
    queries, keys, values and gates.
    """
    for name, t in (("queries", queries), ("keys", keys), ("values", values)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
    if queries.ndim != 3 or keys.ndim != 3 or values.ndim != 3:
        raise ValueError("expected queries (B, N, d_k), keys (E, M, d_k) and values (E, M, C)")
    b, n, dk = queries.shape
    e, m, dkk = keys.shape
    if dkk != dk:
        raise ValueError(f"query/key feature sizes must match; got {dk} and {dkk}")
    if tuple(values.shape[:2]) != (e, m):
        raise ValueError(f"values must be ({e}, {m}, C); got {tuple(values.shape)}")
    if gates is not None:
        if not isinstance(gates, torch.Tensor):
            raise TypeError("gates must be a torch.Tensor")
        if tuple(gates.shape) != (b, n, e):
            raise ValueError(f"expected gates of shape {(b, n, e)}; got {tuple(gates.shape)}")
    if not isinstance(top_k, int) or isinstance(top_k, bool) or not 1 <= top_k <= e * m:
        raise ValueError(f"top_k must be an integer in [1, {e * m}]; got {top_k}")
    if not (queries.dtype == keys.dtype == values.dtype):
        raise ValueError("queries, keys and values must share one dtype")
    if gates is not None and gates.dtype != queries.dtype:
        raise ValueError("gates must have the dtype of the atom projections")
    tensors = (queries, keys, values) + (() if gates is None else (gates,))
    if any(t.device.type != "cuda" or t.device != queries.device for t in tensors):
        raise ValueError("all inputs must be on one CUDA device")
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError("inputs must be contiguous")
    if not isinstance(scale, (int, float)) or isinstance(scale, bool) or not (scale > 0 and scale < float("inf")):
        raise ValueError(f"scale must be a finite positive number; got {scale}")
    _native.load()
    return GatedMixtureFunction.apply(queries, keys, values, gates, top_k, float(scale))
