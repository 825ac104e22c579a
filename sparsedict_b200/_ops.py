"""Tensor-level calls into the C ABI: allocate outputs, launch on the current stream.

Callers own every buffer (the reference convention, outputs made with
``torch.empty``/``torch.zeros``); inputs must already be contiguous.  These
helpers do no argument validation beyond what the C ABI itself rejects —
the public modules validate first, with the reference's messages.
"""

from __future__ import annotations

import torch

from . import _native as nat


_deterministic = False


def set_deterministic_backward(flag: bool) -> None:
    """Choose the backward used for gradients in the input dtype.

    ``False`` (default): the scatter kernel — dK/dV accumulated with fp32
    vector atomics (fastest; summation order, hence the last bits of dK/dV,
    may vary from run to run).  ``True``: the key-major kernels — every
    gradient element written once in a fixed order, bit-identical from run
    to run (bf16/fp16 with d = dv = 64; other shapes always scatter).
    """
    global _deterministic
    _deterministic = bool(flag)


def deterministic_backward() -> bool:
    return _deterministic


def acc_dtype(dtype: torch.dtype) -> torch.dtype:
    """Accumulator / LSE dtype for an input dtype."""
    return torch.float64 if dtype == torch.float64 else torch.float32


def topk_attn_fwd(
    q2: torch.Tensor,
    k2: torch.Tensor,
    v2: torch.Tensor,
    topk: int,
    scale: float,
    *,
    score_grid: int = 0,
    want_scores: bool = False,
    row_offsets: torch.Tensor | None = None,
    row_index: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    seg_bias: torch.Tensor | None = None,
    row_k: torch.Tensor | None = None,
):
    """Fused forward over ``q2 [rows or (S, n), d]``, ``k2 [S, m, d]``, ``v2 [S, m, dv]``.

    Returns ``(out, top_idx int32 [rows, k], lse [rows], top_scores|None)``
    where ``rows`` is ``S * n`` (uniform slices) or the grouped row count.
    ``seg_bias [rows, segs]`` (accumulator dtype, optional) adds
    ``seg_bias[r, j // (m // segs)]`` to the scaled score of row ``r`` and
    key ``j`` (``m`` must divide into ``segs`` equal segments).  ``row_k
    [rows]`` (int32, optional) gives each row its own number of selected keys
    (at most ``topk``; the row's other index slots are -1).
    """
    slices, m, d = k2.shape
    dv = v2.shape[-1]
    if row_offsets is None:
        n = q2.shape[-2]
        rows = slices * n
    else:
        n = rows = q2.reshape(-1, d).shape[0]
    dev = q2.device
    acc = acc_dtype(q2.dtype)
    if out is None:
        out = torch.empty((*q2.shape[:-1], dv), device=dev, dtype=q2.dtype)
    idx = torch.empty((rows, topk), device=dev, dtype=torch.int32)
    lse = torch.empty((rows,), device=dev, dtype=acc)
    scores = torch.empty((rows, topk), device=dev, dtype=acc) if want_scores else None
    with torch.cuda.device(dev):
        head = (q2.data_ptr(), k2.data_ptr(), v2.data_ptr(), out.data_ptr(), idx.data_ptr(), lse.data_ptr(),
                nat.ptr(scores), nat.ptr(row_offsets), nat.ptr(row_index),
                slices, n, m, d, dv, topk, float(scale), int(score_grid))
        if row_k is not None:
            nat.call("sdk_topk_attn_fwd_adaptive", *head, row_k.data_ptr(), nat.TORCH_TO_SDK[q2.dtype],
                     nat.stream_of(dev))
        elif seg_bias is None:
            # scratch from torch's allocator, like every other buffer of the op
            code = nat.TORCH_TO_SDK[q2.dtype]
            nbytes = int(nat.load().sdk_topk_attn_fwd_workspace_size(
                rows, m, d, dv, topk, int(score_grid), int(row_offsets is not None or row_index is not None), code))
            ws = torch.empty((nbytes,), device=dev, dtype=torch.uint8) if nbytes else None
            nat.call("sdk_topk_attn_fwd_ws", *head, code, nat.ptr(ws), nbytes, nat.stream_of(dev))
        else:
            segs = seg_bias.shape[-1]
            nat.call("sdk_topk_attn_fwd_biased", *head, seg_bias.data_ptr(), m // segs, segs,
                     nat.TORCH_TO_SDK[q2.dtype], nat.stream_of(dev))
    return out, idx, lse, scores


def topk_attn_bwd(
    q2: torch.Tensor,
    k2: torch.Tensor,
    v2: torch.Tensor,
    dout2: torch.Tensor,
    top_idx: torch.Tensor,
    lse: torch.Tensor,
    scale: float,
    *,
    score_grid: int = 0,
    dk_acc: torch.Tensor | None = None,
    dv_acc: torch.Tensor | None = None,
    accumulate: bool = False,
    row_offsets: torch.Tensor | None = None,
    row_index: torch.Tensor | None = None,
    dq: torch.Tensor | None = None,
    seg_bias: torch.Tensor | None = None,
    dseg_bias: torch.Tensor | None = None,
):
    """Sparse backward; returns ``(dq, dk_acc, dv_acc)`` (accumulators in ``acc_dtype``).

    With ``seg_bias`` (as in ``topk_attn_fwd``), ``dseg_bias [rows, segs]``
    (optional) receives the per-segment sums of dS over each row's selection.
    """
    slices, m, d = k2.shape
    dv = v2.shape[-1]
    topk = top_idx.shape[-1]
    n = q2.shape[-2] if row_offsets is None else q2.reshape(-1, d).shape[0]
    dev = q2.device
    acc = acc_dtype(q2.dtype)
    if dq is None:
        dq = torch.empty_like(q2)
    if dk_acc is None:
        dk_acc = torch.empty((slices, m, d), device=dev, dtype=acc)
    if dv_acc is None:
        dv_acc = torch.empty((slices, m, dv), device=dev, dtype=acc)
    with torch.cuda.device(dev):
        head = (q2.data_ptr(), k2.data_ptr(), v2.data_ptr(), dout2.data_ptr(), top_idx.data_ptr(), lse.data_ptr(),
                dq.data_ptr(), dk_acc.data_ptr(), dv_acc.data_ptr(), nat.ptr(row_offsets), nat.ptr(row_index),
                slices, n, m, d, dv, topk, float(scale), int(score_grid), int(accumulate))
        if seg_bias is None:
            nat.call("sdk_topk_attn_bwd", *head, nat.TORCH_TO_SDK[q2.dtype], nat.stream_of(dev))
        else:
            segs = seg_bias.shape[-1]
            nat.call("sdk_topk_attn_bwd_biased", *head, seg_bias.data_ptr(), nat.ptr(dseg_bias), m // segs, segs,
                     nat.TORCH_TO_SDK[q2.dtype], nat.stream_of(dev))
    return dq, dk_acc, dv_acc


def topk_attn_bwd_direct(
    q2: torch.Tensor,
    k2: torch.Tensor,
    v2: torch.Tensor,
    dout2: torch.Tensor,
    top_idx: torch.Tensor,
    lse: torch.Tensor,
    scale: float,
    *,
    score_grid: int = 0,
    row_offsets: torch.Tensor | None = None,
    row_index: torch.Tensor | None = None,
    dq: torch.Tensor | None = None,
    dk: torch.Tensor | None = None,
    dv: torch.Tensor | None = None,
    shared_kv: bool = False,
):
    """Backward straight into input-dtype gradients; returns ``(dq, dk, dv)``.

    bf16/fp16 with d = dv = 64 and k <= 64 run the deterministic key-major
    kernels (bit-identical from run to run, no accumulators); other shapes
    scatter into fp32/fp64 accumulators inside the workspace and convert.
    ``shared_kv``: keys and values are one tensor and ``dk`` (= ``dv``)
    receives dK + dV.
    """
    slices, m, d = k2.shape
    dvd = v2.shape[-1]
    topk = top_idx.shape[-1]
    grouped = row_offsets is not None
    n = q2.shape[-2] if not grouped else q2.reshape(-1, d).shape[0]
    rows = n if grouped else slices * n
    dev = q2.device
    if dq is None:
        dq = torch.empty_like(q2)
    if dk is None:
        dk = torch.empty((slices, m, d), device=dev, dtype=q2.dtype)
    if shared_kv:
        dv = dk
    elif dv is None:
        dv = torch.empty((slices, m, dvd), device=dev, dtype=q2.dtype)
    code = nat.TORCH_TO_SDK[q2.dtype]
    lib = nat.load()
    nbytes = int(lib.sdk_topk_attn_bwd_workspace_size(rows, slices, m, d, dvd, topk, int(score_grid), int(grouped),
                                                      code))
    ws = torch.empty((nbytes + 256,), device=dev, dtype=torch.uint8)
    base = ws.data_ptr()
    aligned = (base + 255) // 256 * 256
    with torch.cuda.device(dev):
        nat.call("sdk_topk_attn_bwd_direct", q2.data_ptr(), k2.data_ptr(), v2.data_ptr(), dout2.data_ptr(),
                 top_idx.data_ptr(), lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                 nat.ptr(row_offsets), nat.ptr(row_index), slices, n, m, d, dvd, topk, float(scale),
                 int(score_grid), code, aligned, nbytes, nat.stream_of(dev))
    return dq, dk, dv


def topk_attn_bwd_out(
    q2: torch.Tensor,
    k2: torch.Tensor,
    v2: torch.Tensor,
    dout2: torch.Tensor,
    top_idx: torch.Tensor,
    lse: torch.Tensor,
    scale: float,
    *,
    score_grid: int = 0,
    row_offsets: torch.Tensor | None = None,
    row_index: torch.Tensor | None = None,
    dq: torch.Tensor | None = None,
    dk: torch.Tensor | None = None,
    dv: torch.Tensor | None = None,
    shared_kv: bool = False,
):
    """Backward into input-dtype ``(dq, dk, dv)`` by the selected kernel
    (``set_deterministic_backward``): the key-major kernels, or the scatter
    kernel into fp32/fp64 accumulators followed by one conversion."""
    if _deterministic:
        return topk_attn_bwd_direct(q2, k2, v2, dout2, top_idx, lse, scale, score_grid=score_grid,
                                    row_offsets=row_offsets, row_index=row_index, dq=dq, dk=dk, dv=dv,
                                    shared_kv=shared_kv)
    slices, m, d = k2.shape
    dvd = v2.shape[-1]
    acc = acc_dtype(q2.dtype)
    dk_acc = torch.empty((slices, m, d), device=q2.device, dtype=acc)
    dv_acc = dk_acc if shared_kv else torch.empty((slices, m, dvd), device=q2.device, dtype=acc)
    dq, dk_acc, dv_acc = topk_attn_bwd(q2, k2, v2, dout2, top_idx, lse, scale, score_grid=score_grid,
                                       dk_acc=dk_acc, dv_acc=dv_acc, row_offsets=row_offsets,
                                       row_index=row_index, dq=dq)
    if dk is None:
        dk = torch.empty((slices, m, d), device=q2.device, dtype=q2.dtype)
    finalize_grad(dk_acc, q2.dtype, out=dk)
    if shared_kv:
        return dq, dk, dk
    if dv is None:
        dv = torch.empty((slices, m, dvd), device=q2.device, dtype=q2.dtype)
    finalize_grad(dv_acc, q2.dtype, out=dv)
    return dq, dk, dv


def finalize_grad(acc: torch.Tensor, dtype: torch.dtype, multiplier: float = 1.0,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Accumulator -> ``dtype`` (returns ``acc`` itself when no conversion is needed
    and no ``out`` is given; ``out`` is a contiguous tensor of ``acc``'s shape)."""
    if out is None and acc.dtype == dtype and multiplier == 1.0:
        return acc
    if out is None:
        out = torch.empty(acc.shape, device=acc.device, dtype=dtype)
    with torch.cuda.device(acc.device):
        nat.call("sdk_finalize_grad", acc.data_ptr(), out.data_ptr(), acc.numel(), float(multiplier),
                 nat.TORCH_TO_SDK[dtype], nat.stream_of(acc.device))
    return out


def affinity(queries: torch.Tensor, keys: torch.Tensor) -> torch.Tensor:
    n, d = queries.shape
    m = keys.shape[0]
    scores = torch.empty((n, m), device=queries.device, dtype=torch.float32)
    with torch.cuda.device(queries.device):
        nat.call("sdk_affinity", queries.data_ptr(), keys.data_ptr(), scores.data_ptr(), n, m, d,
                 queries.stride(0), keys.stride(0), nat.TORCH_TO_SDK[queries.dtype], nat.stream_of(queries.device))
    return scores


def select(scores: torch.Tensor, k: int):
    rows, m = scores.shape
    vals = torch.empty((rows, k), device=scores.device, dtype=scores.dtype)
    idx = torch.empty((rows, k), device=scores.device, dtype=torch.int64)
    with torch.cuda.device(scores.device):
        nat.call("sdk_topk_select", scores.data_ptr(), vals.data_ptr(), idx.data_ptr(), rows, m, scores.stride(0),
                 k, nat.TORCH_TO_SDK[scores.dtype], nat.stream_of(scores.device))
    return vals, idx


def aggregate(top_scores: torch.Tensor, top_indices: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
    rows, k = top_scores.shape
    m, dv = values.shape
    out = torch.empty((rows, dv), device=values.device, dtype=torch.float32)
    with torch.cuda.device(values.device):
        nat.call("sdk_topk_aggregate", top_scores.data_ptr(), top_indices.data_ptr(), values.data_ptr(),
                 out.data_ptr(), rows, k, m, dv, top_scores.stride(0), top_indices.stride(0), values.stride(0),
                 nat.TORCH_TO_SDK[top_scores.dtype], 64 if top_indices.dtype == torch.int64 else 32,
                 nat.TORCH_TO_SDK[values.dtype], nat.stream_of(values.device))
    return out


def route_top1(logits: torch.Tensor):
    """Top-1 routing: ``(expert [n], order [n], offsets [E+1])`` as int32 device tensors."""
    n, experts = logits.shape
    dev = logits.device
    expert = torch.empty((n,), device=dev, dtype=torch.int32)
    order = torch.empty((n,), device=dev, dtype=torch.int32)
    offsets = torch.empty((experts + 1,), device=dev, dtype=torch.int32)
    with torch.cuda.device(dev):
        nat.call("sdk_route_top1", logits.data_ptr(), n, experts, expert.data_ptr(), order.data_ptr(),
                 offsets.data_ptr(), nat.stream_of(dev))
    return expert, order, offsets
