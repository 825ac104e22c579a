"""Fused top-k sparse attention on B200: the drop-in for SparseDict's
``kernels/fused_topk_attn.py``.

Same public names, signatures, saved tensors and ``ValueError`` messages as
the reference module (``fused_topk_attention`` :1204-1289,
``FusedTopKAttentionFunction`` :980-1201, ``tiled_affinity`` :227-287,
``tiled_topk`` :290-336, ``tiled_topk_aggregate`` :339-408).  Underneath,
every stage runs in the hand-written sm_100a kernels of
``libsparsedict_b200.so``; there is no Triton and no CPU fallback.  Beyond
the reference, bfloat16 and float16 inputs are accepted (fp32 accumulation,
output in the input dtype).
"""

from __future__ import annotations

import math

import torch

from .. import _native, _ops

_FUSED_DTYPE_MESSAGE = "fused path supports float32, float64, bfloat16 and float16 inputs"
_FUSED_DTYPES = (torch.float32, torch.float64, torch.bfloat16, torch.float16)


def _require_native(op: str) -> None:
    if not _native.available():
        raise RuntimeError(
            f"the sparsedict_b200 native library is required for {op}; build it with "
            "`python -m sparsedict_b200.build`"
        )


def tiled_affinity(queries: torch.Tensor, keys: torch.Tensor) -> torch.Tensor:
    """Dense ``queries @ keys.T`` in float32 for ``(N, D)`` / ``(M, D)`` inputs."""
    if queries.ndim != 2 or keys.ndim != 2:
        raise ValueError("queries and keys must be rank-2 (items, features) tensors")
    if queries.size(1) != keys.size(1):
        raise ValueError(
            f"query/key feature sizes must match; got {queries.size(1)} and {keys.size(1)}"
        )
    if queries.size(0) == 0 or keys.size(0) == 0 or queries.size(1) == 0:
        raise ValueError("query, key, and feature dimensions must be non-empty")
    if queries.stride(1) != 1 or keys.stride(1) != 1:
        raise ValueError("query and key feature dimensions must be contiguous")
    if queries.device.type != "cuda" or keys.device.type != "cuda":
        raise ValueError("tiled_affinity requires CUDA query and key tensors")
    if queries.device != keys.device:
        raise ValueError("queries and keys must be on the same CUDA device")
    if queries.dtype != keys.dtype or queries.dtype not in (torch.float16, torch.float32):
        raise ValueError("queries and keys must share a float16 or float32 dtype")
    _require_native("tiled_affinity")
    return _ops.affinity(queries, keys)


def tiled_topk(scores: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Each row's ``k`` largest scores (input dtype) and their int64 indices.

    Equal scores are ordered by ascending column index and NaN ranks above
    every number, so index order is fully determined, ties included.
    """
    if scores.ndim != 2:
        raise ValueError("scores must be a rank-2 (queries, keys) tensor")
    if scores.size(0) == 0 or scores.size(1) == 0:
        raise ValueError("score dimensions must be non-empty")
    if not isinstance(k, int) or isinstance(k, bool) or not 1 <= k <= scores.size(1):
        raise ValueError(f"k must be an integer in [1, {scores.size(1)}]")
    if scores.device.type != "cuda":
        raise ValueError("tiled_topk requires CUDA scores")
    if scores.dtype not in (torch.float16, torch.float32):
        raise ValueError("scores must have float16 or float32 dtype")
    if scores.stride(1) != 1:
        scores = scores.contiguous()
    _require_native("tiled_topk")
    return _ops.select(scores, k)


def tiled_topk_aggregate(
    top_scores: torch.Tensor,
    top_indices: torch.Tensor,
    values: torch.Tensor,
) -> torch.Tensor:
    """Softmax-weight the gathered value rows of each query's selected keys (float32 out)."""
    if top_scores.ndim != 2 or top_indices.ndim != 2:
        raise ValueError("top_scores and top_indices must be rank-2 tensors")
    if values.ndim != 2:
        raise ValueError("values must be a rank-2 (keys, features) tensor")
    if top_scores.shape != top_indices.shape:
        raise ValueError("top_scores and top_indices must have identical shapes")
    if top_scores.size(0) == 0 or top_scores.size(1) == 0 or values.size(1) == 0:
        raise ValueError("query, top-k, and value feature dimensions must be non-empty")
    if values.size(0) == 0:
        raise ValueError("values must contain at least one key row")
    if top_scores.device.type != "cuda" or top_indices.device.type != "cuda":
        raise ValueError("tiled_topk_aggregate requires CUDA tensors")
    if values.device.type != "cuda":
        raise ValueError("tiled_topk_aggregate requires CUDA values")
    if top_scores.device != top_indices.device or top_scores.device != values.device:
        raise ValueError("scores, indices, and values must be on the same CUDA device")
    if top_scores.dtype not in (torch.float16, torch.float32):
        raise ValueError("top_scores must have float16 or float32 dtype")
    if values.dtype not in (torch.float16, torch.float32):
        raise ValueError("values must have float16 or float32 dtype")
    if top_indices.dtype not in (torch.int32, torch.int64):
        raise ValueError("top_indices must have int32 or int64 dtype")
    if top_scores.stride(1) != 1 or top_indices.stride(1) != 1:
        raise ValueError("top-k dimensions must be contiguous")
    if values.stride(1) != 1:
        raise ValueError("value feature dimension must be contiguous")
    _require_native("tiled_topk_aggregate")
    return _ops.aggregate(top_scores, top_indices, values)


class FusedTopKAttentionFunction(torch.autograd.Function):
    """Top-k attention with a fused sm_100a forward and a sparse backward.

    Forward: one kernel computes the scaled affinity tile by tile, keeps each
    row's top-k without writing the score row to memory, and aggregates the
    selected value rows.  Saved for backward: the flattened inputs, the int32
    support indices and the row log-sum-exp — exactly the reference's
    ``ctx.save_for_backward(queries2, keys2, values2, top_indices, lse)``.
    Backward: recomputes the selected scores on that support, writes dQ once
    per row and scatters dK/dV.
    """

    @staticmethod
    def forward(ctx, queries, keys, values, k, temperature=1.0, score_grid=0):
        batch, heads, query_count, feat_q = queries.shape
        key_count = keys.shape[2]
        feat_v = values.shape[3]
        batch_heads = batch * heads
        score_scale = 1.0 / (temperature * math.sqrt(feat_q))

        queries2 = queries.reshape(batch_heads, query_count, feat_q)
        keys2 = keys.reshape(batch_heads, key_count, feat_q)
        values2 = values.reshape(batch_heads, key_count, feat_v)
        out, top_indices, lse, _ = _ops.topk_attn_fwd(
            queries2, keys2, values2, k, score_scale, score_grid=score_grid
        )
        top_indices = top_indices.view(batch_heads, query_count, k)
        lse = lse.view(batch_heads, query_count)
        ctx.save_for_backward(queries2, keys2, values2, top_indices, lse)
        ctx.fused_geometry = (
            batch, heads, query_count, feat_q, key_count, feat_v, k, score_scale, score_grid
        )
        return out.view(batch, heads, query_count, feat_v)

    @staticmethod
    def backward(ctx, grad_output):
        queries2, keys2, values2, top_indices, lse = ctx.saved_tensors
        (batch, heads, query_count, feat_q, key_count, feat_v, k, score_scale, score_grid) = ctx.fused_geometry
        batch_heads = batch * heads
        dtype = queries2.dtype
        grad_output2 = grad_output.reshape(batch_heads, query_count, feat_v).to(dtype).contiguous()
        dq, d_keys, d_values = _ops.topk_attn_bwd_out(
            queries2, keys2, values2, grad_output2, top_indices, lse, score_scale, score_grid=score_grid,
        )
        grads = (
            dq.view(batch, heads, query_count, feat_q),
            d_keys.view(batch, heads, key_count, feat_q),
            d_values.view(batch, heads, key_count, feat_v),
        )
        # k, temperature (and the optional tie-stress grid) get no gradient
        return grads + (None,) * (len(ctx.needs_input_grad) - 3)


def validate_fused_inputs(queries, keys, values, k, temperature) -> None:
    """The reference wrapper's checks (kernels/fused_topk_attn.py:1218-1281), plus bf16/fp16."""
    for name, tensor in (("queries", queries), ("keys", keys), ("values", values)):
        if tensor.ndim != 4:
            raise ValueError(
                f"{name} must be rank-4 (B, H, tokens/atoms, features); got {tuple(tensor.shape)}"
            )
        if not tensor.is_floating_point():
            raise ValueError(f"{name} must have a floating-point dtype; got {tensor.dtype}")
        if tensor.dtype not in _FUSED_DTYPES:
            raise ValueError(_FUSED_DTYPE_MESSAGE)
        if not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if queries.dtype != keys.dtype or queries.dtype != values.dtype:
        raise ValueError("queries, keys, and values must share one dtype")
    if queries.shape[0] != keys.shape[0] or queries.shape[1] != keys.shape[1]:
        raise ValueError("queries and keys must share leading (B, H) dimensions")
    if queries.shape[0:2] != values.shape[0:2]:
        raise ValueError(
            f"queries shape {tuple(queries.shape)} and values shape "
            f"{tuple(values.shape)} must share leading (B, H) dimensions"
        )
    if keys.shape[0:2] != values.shape[0:2]:
        raise ValueError(
            f"keys shape {tuple(keys.shape)} and values shape "
            f"{tuple(values.shape)} must share leading (B, H) dimensions"
        )
    if queries.shape[3] != keys.shape[3]:
        raise ValueError(
            f"query/key feature sizes must match; got {queries.shape[3]} and {keys.shape[3]}"
        )
    if keys.shape[2] != values.shape[2]:
        raise ValueError(
            f"key/value atom counts must match; got {keys.shape[2]} and {values.shape[2]}"
        )
    if queries.shape[0] == 0 or queries.shape[1] == 0:
        raise ValueError("batch and head dimensions must be non-empty")
    if queries.shape[2] == 0 or keys.shape[2] == 0 or queries.shape[3] == 0:
        raise ValueError("query, key, and feature dimensions must be non-empty")
    if values.shape[3] == 0:
        raise ValueError("value feature dimension must be non-empty")
    if not isinstance(k, int) or isinstance(k, bool) or not 1 <= k <= keys.shape[2]:
        raise ValueError(f"k must be an integer in [1, {keys.shape[2]}]; got {k}")
    if not isinstance(temperature, (int, float)) or isinstance(temperature, bool):
        raise ValueError("temperature must be a positive finite number")
    if not math.isfinite(temperature) or temperature <= 0:
        raise ValueError("temperature must be a positive finite number")
    if queries.device.type != "cuda" or keys.device.type != "cuda" or values.device.type != "cuda":
        raise ValueError("fused path requires CUDA tensors")
    if queries.device != keys.device or queries.device != values.device:
        raise ValueError("queries, keys, and values must be on the same device")


def fused_topk_attention(
    queries: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    k: int,
    temperature: float = 1.0,
) -> torch.Tensor:
    """Fused CUDA sparse top-k cross attention returning ``(B, H, N, d_v)``.

    Scores are scaled by ``1 / (temperature * sqrt(d_k))``.  Inputs must
    share leading ``(B, H)`` dimensions and be contiguous CUDA tensors of one
    dtype (float32, float64, bfloat16 or float16).  Raises ``ValueError``
    with the reference's messages for invalid geometry or temperature.
    """
    validate_fused_inputs(queries, keys, values, k, temperature)
    _require_native("fused_topk_attention")
    limit = _native.max_topk(queries.dtype, queries.shape[3])
    if k > limit:
        raise ValueError(
            f"k={k} exceeds the fused kernel's per-row capacity of {limit} for "
            f"feature size {queries.shape[3]} and {queries.dtype}"
        )
    return FusedTopKAttentionFunction.apply(queries, keys, values, k, float(temperature))
