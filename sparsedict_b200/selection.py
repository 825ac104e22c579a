"""SparseDict's top-k selection operators, with the selection on the GPU.

``models/modules/topk_select.py`` (SparseDict): ``hard_topk_mask``,
``straight_through_topk``, ``gumbel_perturbed_topk`` and
``sparse_topk_attention`` with ``selection="hard"`` or ``"ste"``, over a given
score tensor ``(..., Q, M)``.  Same names, arguments, results and error
messages.  The per-row top-k runs in the select kernel (``sdk_topk_select``:
descending score, lower index on ties, NaN first; exact for fp32, fp16, bf16
and fp64); the softmax over the selected scores, the dense weights and masked
scores and the weighted sum of the gathered value rows run in one warp-per-row
kernel (``sdk_sparse_topk_attn_fwd``), their gradient in another
(``sdk_sparse_topk_attn_bwd``), and the masks in ``sdk_fill_scatter``.  Both
selection modes route a selected score's gradient to that score only
(``topk_select.py:33-45``; ``torch.topk`` does the same for ``"hard"``), so
they differ in name only.

The fused kernels (``fused_topk_attention``) never materialise the dense
scores; these operators exist for callers that already hold them.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import torch

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


def _fill_scatter(src: torch.Tensor, idx: torch.Tensor, shape, fill: float) -> torch.Tensor:
    """Dense ``shape`` tensor of ``fill`` with ``src`` at ``idx`` along the last axis (native kernel)."""
    out = torch.empty(shape, dtype=src.dtype, device=src.device)
    k = idx.size(-1)
    rows = idx.numel() // k
    src_c, idx_c = src.contiguous(), idx.contiguous()
    with torch.cuda.device(src.device):
        _native.call("sdk_fill_scatter", src_c.data_ptr(), idx_c.data_ptr(), out.data_ptr(), rows, k, shape[-1],
                     float(fill), _native.TORCH_TO_SDK[src.dtype], _native.stream_of(src.device))
    return out


class _StraightThroughTopK(torch.autograd.Function):
    """Top-k whose gradient reaches the selected scores only."""

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
        return _fill_scatter(grad_vals, idx, ctx.input_shape, 0.0), None


class _MaskSelected(torch.autograd.Function):
    """``-inf`` everywhere but the selected scores (gradient: the selected entries)."""

    @staticmethod
    def forward(ctx, vals, idx, shape):
        ctx.save_for_backward(idx)
        return _fill_scatter(vals, idx, shape, float("-inf"))

    @staticmethod
    def backward(ctx, grad):
        (idx,) = ctx.saved_tensors
        return grad.gather(-1, idx), None, None


def straight_through_topk(scores: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Sorted top-k scores and int64 indices with selected-only gradients."""
    _validate_scores(scores, k)
    return _StraightThroughTopK.apply(scores, k)


def hard_topk_mask(scores: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """All but the top-k scores set to ``-inf`` along the last axis, and the indices."""
    _validate_scores(scores, k)
    vals, idx = _StraightThroughTopK.apply(scores, k)
    return _MaskSelected.apply(vals, idx, scores.shape), idx


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


class _SparseTopKAttention(torch.autograd.Function):
    """Selection, softmax, dense weights and masked scores, and the value sum, on the
    native kernels; the gradient reaches the selected scores and the gathered
    value rows.  ``values`` is already in the output dtype."""

    @staticmethod
    def forward(ctx, scores, values, k):
        vals, idx = _select(scores, k)
        shape = scores.shape
        q, m = shape[-2], shape[-1]
        rows = idx.numel() // k
        rpb = q if values.ndim > 2 else 0
        dv = values.size(-1)
        dev = scores.device
        out = torch.empty((*shape[:-1], dv), dtype=values.dtype, device=dev)
        weights = torch.empty(shape, dtype=scores.dtype, device=dev)
        masked = torch.empty(shape, dtype=scores.dtype, device=dev)
        values_c = values.contiguous()
        with torch.cuda.device(dev):
            _native.call("sdk_sparse_topk_attn_fwd", vals.data_ptr(), idx.data_ptr(), values_c.data_ptr(),
                         out.data_ptr(), weights.data_ptr(), masked.data_ptr(), rows, rpb, k, m, dv,
                         _native.TORCH_TO_SDK[scores.dtype], _native.TORCH_TO_SDK[values.dtype],
                         _native.stream_of(dev))
        ctx.save_for_backward(vals, idx, values_c)
        ctx.geometry = (shape, rows, rpb, k, m, dv)
        ctx.mark_non_differentiable(idx)
        return out, weights, idx, masked

    @staticmethod
    def backward(ctx, g_out, g_weights, g_idx, g_masked):
        vals, idx, values = ctx.saved_tensors
        shape, rows, rpb, k, m, dv = ctx.geometry
        dev = vals.device
        if g_out is None:
            g_out = torch.zeros((*shape[:-1], dv), dtype=values.dtype, device=dev)
        g_out = g_out.contiguous()
        g_weights = None if g_weights is None else g_weights.contiguous()
        g_masked = None if g_masked is None else g_masked.contiguous()
        g_scores = torch.empty(shape, dtype=vals.dtype, device=dev)
        acc = torch.float64 if values.dtype == torch.float64 else torch.float32
        g_values = torch.zeros(values.shape, dtype=acc, device=dev)
        with torch.cuda.device(dev):
            _native.call("sdk_sparse_topk_attn_bwd", vals.data_ptr(), idx.data_ptr(), values.data_ptr(),
                         g_out.data_ptr(), _native.ptr(g_weights), _native.ptr(g_masked), g_scores.data_ptr(),
                         g_values.data_ptr(), rows, rpb, k, m, dv, _native.TORCH_TO_SDK[vals.dtype],
                         _native.TORCH_TO_SDK[values.dtype], _native.stream_of(dev))
        return g_scores, g_values.to(values.dtype), None


def sparse_topk_attention(
    scores: torch.Tensor,
    values: torch.Tensor,
    k: int,
    selection: str = "hard",
) -> TopKAttentionResult:
    """Softmax over each row's top-k scores and the weighted sum of the selected value rows.

    ``values`` is shared ``(M, D)`` or batch-specific ``(..., M, D)``.  Returns
    the reference's ``TopKAttentionResult(output, weights, indices,
    masked_scores)`` (``topk_select.py:106-162``) with its argument checks and
    messages; the output has the promoted dtype of scores and values.  Both
    selection modes have the same forward and gradient.
    """
    if selection not in ("hard", "ste"):
        raise ValueError(f"selection must be 'hard' or 'ste'; got {selection!r}")
    _validate_scores(scores, k)
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
    if k > 256:
        raise ValueError(f"k must be at most 256 on this path; got {k}")
    out_dtype = torch.promote_types(scores.dtype, values.dtype)
    output, weights, indices, masked = _SparseTopKAttention.apply(scores, values.to(out_dtype), k)
    return TopKAttentionResult(output, weights, indices, masked)
