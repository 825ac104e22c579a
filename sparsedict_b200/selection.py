"""SparseDict's top-k selection operators, with the selection on the GPU.

``models/modules/topk_select.py`` (SparseDict): ``hard_topk_mask``,
``straight_through_topk``, ``gumbel_perturbed_topk`` and
``sparse_topk_attention`` with ``selection="hard"`` or ``"ste"``, over a given
score tensor ``(..., Q, M)``.  Same names, arguments, results and error
messages.  The per-row top-k runs in the select kernel (``sdk_topk_select``:
descending score, lower index on ties, NaN first; exact for fp32, fp16, bf16
and fp64); the small ``(..., Q, k)`` softmax/gather that follows is the
reference's own formula.  Both selection modes route a selected score's
gradient to that score only (``topk_select.py:33-45``; ``torch.topk`` does the
same for ``"hard"``), so they differ in name only.

The fused kernels (``fused_topk_attention``) never materialise the dense
scores; these operators exist for callers that already hold them.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import torch
import torch.nn.functional as F

from . import _native, _ops


class TopKAttentionResult(NamedTuple):
    output: torch.Tensor
    weights: torch.Tensor
    indices: torch.Tensor
    masked_scores: torch.Tensor


def _validate_scores(scores: torch.Tensor, k: int) -> None:
    # models/modules/topk_select.py:165-173
    if scores.ndim < 2:
        raise ValueError(f"expected scores with query and atom dimensions, got {tuple(scores.shape)}")
    if not scores.is_floating_point():
        raise ValueError("scores must have a floating-point dtype")
    if not 1 <= k <= scores.size(-1):
        raise ValueError(f"k must be between 1 and {scores.size(-1)}; got {k}")
    if scores.device.type != "cuda":
        raise ValueError("scores must be a CUDA tensor")
    _native.load()


def _select(scores: torch.Tensor, k: int):
    m = scores.size(-1)
    flat = scores.detach().reshape(-1, m).contiguous()
    vals, idx = _ops.select(flat, k)
    return vals.reshape(*scores.shape[:-1], k), idx.reshape(*scores.shape[:-1], k)


class _StraightThroughTopK(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scores, k):
        vals, idx = _select(scores, k)
        ctx.save_for_backward(idx)
        ctx.input_shape = scores.shape
        ctx.mark_non_differentiable(idx)
        return vals, idx

    @staticmethod
    def backward(ctx, grad_vals, grad_idx):
        if grad_vals is None:
            return None, None
        (idx,) = ctx.saved_tensors
        return grad_vals.new_zeros(ctx.input_shape).scatter(-1, idx, grad_vals), None


def straight_through_topk(scores: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Sorted top-k scores and int64 indices with selected-only gradients."""
    _validate_scores(scores, k)
    return _StraightThroughTopK.apply(scores, k)


def hard_topk_mask(scores: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """All but the top-k scores set to ``-inf`` along the last axis, and the indices."""
    _validate_scores(scores, k)
    vals, idx = _StraightThroughTopK.apply(scores, k)
    return torch.full_like(scores, float("-inf")).scatter(-1, idx, vals), idx


def gumbel_perturbed_topk(
    scores: torch.Tensor,
    k: int,
    sigma: float = 1.0,
    num_samples: int = 2,
    generator: torch.Generator | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Monte Carlo top-k samples under Gumbel perturbation (leading sample axis).

    The noise is drawn exactly as ``topk_select.py:75-88`` draws it (one
    ``torch.rand`` of the score shape per sample, clamped to
    ``[eps, 1 - eps]``, ``-log(-log(u))``), so the same generator state gives
    the reference's samples.  Gradients reach the base scores of the entries
    each sample selected.
    """
    _validate_scores(scores, k)
    if sigma < 0 or not math.isfinite(sigma):
        raise ValueError(f"sigma must be finite and non-negative; got {sigma}")
    if num_samples <= 0:
        raise ValueError(f"num_samples must be positive; got {num_samples}")
    eps = torch.finfo(scores.dtype).eps
    vals, idxs = [], []
    for _ in range(num_samples):
        u = torch.rand(scores.shape, dtype=scores.dtype, device=scores.device, generator=generator)
        noise = -torch.log(-torch.log(u.clamp(min=eps, max=1.0 - eps)))
        v, i = straight_through_topk(scores + sigma * noise, k)
        vals.append(v)
        idxs.append(i)
    return torch.stack(vals), torch.stack(idxs)


def sparse_topk_attention(
    scores: torch.Tensor,
    values: torch.Tensor,
    k: int,
    selection: str = "hard",
) -> TopKAttentionResult:
    """Softmax over each row's top-k scores and the weighted sum of the selected value rows.

    ``values`` is shared ``(M, D)`` or batch-specific ``(..., M, D)``.  Returns
    the reference's ``TopKAttentionResult(output, weights, indices,
    masked_scores)`` (``topk_select.py:106-162``).
    """
    if selection == "hard":
        masked_scores, indices = hard_topk_mask(scores, k)
    elif selection == "ste":
        selected, indices = straight_through_topk(scores, k)
        masked_scores = torch.full_like(scores, float("-inf")).scatter(-1, indices, selected)
    else:
        raise ValueError(f"selection must be 'hard' or 'ste'; got {selection!r}")
    if values.ndim < 2:
        raise ValueError(f"expected values with atom and feature dimensions, got {tuple(values.shape)}")
    if values.size(-2) != scores.size(-1):
        raise ValueError(f"value atom count {values.size(-2)} must match score width {scores.size(-1)}")
    if values.device != scores.device:
        raise ValueError("scores and values must be on the same device")
    batch_shape = scores.shape[:-2]
    value_batch_shape = values.shape[:-2]
    if value_batch_shape and tuple(value_batch_shape) != tuple(batch_shape):
        raise ValueError(
            "values must be shared across batches or have leading dimensions "
            f"{tuple(batch_shape)}; got {tuple(value_batch_shape)}"
        )
    selected_weights = F.softmax(masked_scores.gather(-1, indices), dim=-1)
    weights = torch.zeros_like(scores).scatter(-1, indices, selected_weights)
    q = scores.size(-2)
    expanded = values.unsqueeze(-3).expand(*batch_shape, q, values.size(-2), values.size(-1))
    selected_values = expanded.gather(-2, indices.unsqueeze(-1).expand(*indices.shape, values.size(-1)))
    output = (selected_values * selected_weights.unsqueeze(-1)).sum(dim=-2)
    return TopKAttentionResult(output, weights, indices, masked_scores)
