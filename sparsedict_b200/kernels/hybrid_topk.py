"""Drop-in for SparseDict's ``kernels/hybrid_topk.py`` on B200.

The reference's "hybrid" forward (chunked cuBLAS scores written to memory,
chunk-local ``torch.topk``, a Triton merge/softmax/gather kernel,
``kernels/hybrid_topk.py:153-290``) is served here by the same fused sm_100a
kernel as ``fused_topk_attention``: no score chunk is written to memory.  The
public names, argument checks, messages and return layout are the
reference's (``_hybrid_topk_attention_with_aux`` :153-290,
``hybrid_topk_attention`` :293-319).
"""

from __future__ import annotations

import math

import torch

from .. import _native, _ops

_HYBRID_DTYPE_MESSAGE = "hybrid path supports float32 inputs"


def _hybrid_topk_attention_with_aux(
    queries: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    k: int,
    score_scale: float,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Return ``(top_scores, top_indices int32, lse, out)`` for the autograd wrapper."""
    if not all(torch.is_tensor(tensor) for tensor in (queries, keys, values)):
        raise TypeError("queries, keys, and values must be torch tensors")
    if queries.ndim != 4 or keys.ndim != 4 or values.ndim != 4:
        raise ValueError("queries/keys/values must be rank-4 (B, H, N, D)")
    if not all(tensor.is_contiguous() for tensor in (queries, keys, values)):
        raise ValueError("queries, keys, and values must be contiguous")
    if (
        queries.device.type != "cuda"
        or keys.device != queries.device
        or values.device != queries.device
    ):
        raise ValueError("queries, keys, and values must share a CUDA device")
    if any(tensor.dtype != torch.float32 for tensor in (queries, keys, values)):
        raise ValueError(_HYBRID_DTYPE_MESSAGE)
    if not isinstance(k, int) or isinstance(k, bool) or k < 1:
        raise ValueError("k must be a positive integer")
    if not _native.available():
        raise RuntimeError(
            "hybrid path requires the sparsedict_b200 native library; build it with "
            "`python -m sparsedict_b200.build`"
        )
    batch, heads, query_count, feat_q = queries.shape
    key_count = keys.shape[2]
    feat_v = values.shape[3]
    if k >= key_count:
        raise ValueError(f"hybrid selector requires k in [1, {key_count - 1}]")
    if (batch, heads) != keys.shape[:2] or (batch, heads) != values.shape[:2]:
        raise ValueError("queries, keys, and values must share batch and head dimensions")
    if queries.shape[3] != keys.shape[3]:
        raise ValueError("query and key feature dimensions must match")
    if key_count != values.shape[2]:
        raise ValueError("key and value atom counts must match")
    if min(batch, heads, query_count, key_count, feat_q, feat_v) <= 0:
        raise ValueError("batch, token, key, and feature dimensions must be non-empty")
    limit = _native.max_topk(torch.float32, feat_q)
    if k > limit:
        raise ValueError(f"k={k} exceeds the fused kernel's per-row capacity of {limit}")

    batch_heads = batch * heads
    queries2 = queries.reshape(batch_heads, query_count, feat_q)
    keys2 = keys.reshape(batch_heads, key_count, feat_q)
    values2 = values.reshape(batch_heads, key_count, feat_v)
    out, top_indices, lse, top_scores = _ops.topk_attn_fwd(
        queries2, keys2, values2, k, score_scale, want_scores=True
    )
    return (
        top_scores.reshape(batch_heads, query_count, k),
        top_indices.reshape(batch_heads, query_count, k),
        lse.reshape(batch_heads, query_count),
        out.reshape(batch_heads, query_count, feat_v),
    )


def hybrid_topk_attention(
    queries: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    k: int,
    temperature: float = 1.0,
) -> torch.Tensor:
    """Forward-only float32 top-k attention; ``k == M`` delegates to the fused op."""
    if not torch.is_tensor(queries):
        raise TypeError("queries, keys, and values must be torch tensors")
    if not torch.is_tensor(keys) or keys.ndim != 4:
        raise ValueError("keys must be rank-4 (B, H, M, D)")
    if queries.ndim != 4:
        raise ValueError("queries must be rank-4 (B, H, N, D)")
    if not isinstance(temperature, (int, float)) or isinstance(temperature, bool):
        raise ValueError("temperature must be a positive finite number")
    if not math.isfinite(temperature) or temperature <= 0:
        raise ValueError("temperature must be a positive finite number")
    if k == keys.shape[2]:
        from .fused_topk_attn import fused_topk_attention

        return fused_topk_attention(queries, keys, values, k, temperature)
    score_scale = 1.0 / (temperature * math.sqrt(queries.shape[-1]))
    output = _hybrid_topk_attention_with_aux(queries, keys, values, k, score_scale)[-1]
    return output.reshape(*queries.shape[:3], values.shape[-1])
