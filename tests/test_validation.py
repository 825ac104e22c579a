"""CPU-runnable argument checks; messages follow the reference's own tests
(tests/test_triton_autograd.py:206-230, tests/test_fused_topk_attn.py:11-85,
tests/test_hybrid_topk.py:296-302)."""

import pytest
import torch

from sparsedict_b200 import (
    fused_topk_attention,
    hybrid_topk_attention,
    tiled_affinity,
    tiled_topk,
    tiled_topk_aggregate,
)
from sparsedict_b200.kernels.hybrid_topk import _hybrid_topk_attention_with_aux


def test_wrapper_requires_cuda_tensors():
    with pytest.raises(ValueError, match="requires CUDA"):
        fused_topk_attention(torch.rand(1, 1, 4, 2), torch.rand(1, 1, 5, 2), torch.rand(1, 1, 5, 3), 2)


@pytest.mark.parametrize(
    ("queries", "keys", "values", "k", "message"),
    [
        (torch.rand(1, 4, 2), torch.rand(5, 2), torch.rand(5, 3), 2, "rank-4"),
        (torch.rand(1, 2, 4, 2), torch.rand(1, 2, 5, 3), torch.rand(1, 2, 5, 3), 2, "feature sizes must match"),
        (torch.rand(1, 2, 4, 2), torch.rand(1, 2, 5, 2), torch.rand(1, 2, 6, 3), 2, "key/value atom counts must match"),
        (torch.rand(1, 2, 4, 2), torch.rand(1, 2, 5, 2), torch.rand(1, 2, 5, 3), 6, r"k must be an integer"),
        (torch.rand(1, 2, 4, 2), torch.rand(1, 2, 5, 2), torch.rand(1, 2, 5, 3), 0, r"k must be an integer"),
        (torch.rand(1, 2, 4, 2), torch.rand(1, 2, 5, 2), torch.rand(1, 2, 5, 3), True, r"k must be an integer"),
        (torch.rand(1, 2, 4, 2), torch.rand(1, 2, 5, 2), torch.rand(1, 2, 5, 3), 2, "requires CUDA"),
        (torch.rand(1, 2, 4, 2), torch.rand(2, 2, 5, 2), torch.rand(2, 2, 5, 3), 2, "leading"),
        (torch.rand(1, 2, 4, 2).int(), torch.rand(1, 2, 5, 2), torch.rand(1, 2, 5, 3), 2, "floating-point"),
        (torch.rand(1, 2, 2, 4).transpose(2, 3), torch.rand(1, 2, 5, 2), torch.rand(1, 2, 5, 3), 2, "contiguous"),
        (torch.rand(1, 2, 4, 2), torch.rand(1, 2, 5, 2, dtype=torch.float64), torch.rand(1, 2, 5, 3), 2, "one dtype"),
        (torch.rand(1, 0, 4, 2), torch.rand(1, 0, 5, 2), torch.rand(1, 0, 5, 3), 2, "non-empty"),
    ],
)
def test_wrapper_rejects_invalid_geometry(queries, keys, values, k, message):
    with pytest.raises(ValueError, match=message):
        fused_topk_attention(queries, keys, values, k)


@pytest.mark.parametrize("temperature", [0.0, -1.0, float("inf"), float("nan"), True, "1"])
def test_wrapper_rejects_bad_temperature(temperature):
    with pytest.raises(ValueError, match="temperature must be a positive finite number"):
        fused_topk_attention(torch.rand(1, 1, 4, 2), torch.rand(1, 1, 5, 2), torch.rand(1, 1, 5, 3), 2, temperature)


def test_wrapper_rejects_integer_dtype_message():
    q = torch.rand(1, 1, 4, 2).to(torch.int8)
    with pytest.raises(ValueError, match="floating-point dtype"):
        fused_topk_attention(q, q, q, 1)


def test_hybrid_wrapper_requires_cuda():
    with pytest.raises(ValueError, match="share a CUDA device"):
        hybrid_topk_attention(torch.rand(1, 1, 3, 4), torch.rand(1, 1, 5, 4), torch.rand(1, 1, 5, 2), 2)


def test_hybrid_aux_type_and_rank_checks():
    with pytest.raises(TypeError, match="torch tensors"):
        _hybrid_topk_attention_with_aux([1], torch.rand(1, 1, 5, 4), torch.rand(1, 1, 5, 2), 2, 1.0)
    with pytest.raises(ValueError, match="rank-4"):
        _hybrid_topk_attention_with_aux(torch.rand(1, 3, 4), torch.rand(1, 1, 5, 4), torch.rand(1, 1, 5, 2), 2, 1.0)
    with pytest.raises(TypeError):
        hybrid_topk_attention([1], torch.rand(1, 1, 5, 4), torch.rand(1, 1, 5, 2), 2)
    with pytest.raises(ValueError, match="keys must be rank-4"):
        hybrid_topk_attention(torch.rand(1, 1, 3, 4), torch.rand(5, 4), torch.rand(1, 1, 5, 2), 2)


def test_tiled_affinity_rejects_non_matrix_inputs():
    with pytest.raises(ValueError, match="rank-2"):
        tiled_affinity(torch.rand(2, 3, 4), torch.rand(5, 4))


def test_tiled_affinity_rejects_mismatched_features():
    with pytest.raises(ValueError, match="feature sizes must match"):
        tiled_affinity(torch.rand(2, 3), torch.rand(5, 4))


def test_tiled_affinity_requires_contiguous_feature_dimension():
    with pytest.raises(ValueError, match="feature dimensions must be contiguous"):
        tiled_affinity(torch.rand(4, 2).T, torch.rand(5, 4))


def test_tiled_affinity_requires_cuda():
    with pytest.raises(ValueError, match="requires CUDA"):
        tiled_affinity(torch.rand(2, 4), torch.rand(5, 4))


@pytest.mark.parametrize(("shape", "k"), [((1, 1), 1), ((7, 64), 5), ((65, 129), 17), ((8, 256), 64), ((3, 73), 73)])
def test_tiled_topk_rejects_non_cuda_scores(shape, k):
    with pytest.raises(ValueError, match="requires CUDA"):
        tiled_topk(torch.rand(shape), k)


@pytest.mark.parametrize(
    ("scores", "k", "message"),
    [
        (torch.rand(2, 3, 4), 2, "rank-2"),
        (torch.empty(0, 4), 2, "dimensions must be non-empty"),
        (torch.rand(2, 4), 0, r"k must be an integer"),
        (torch.rand(2, 4), 5, r"k must be an integer"),
    ],
)
def test_tiled_topk_rejects_invalid_inputs(scores, k, message):
    with pytest.raises(ValueError, match=message):
        tiled_topk(scores, k)


def test_tiled_topk_aggregate_rejects_incompatible_shapes():
    with pytest.raises(ValueError, match="identical shapes"):
        tiled_topk_aggregate(torch.rand(2, 3), torch.zeros(2, 4, dtype=torch.int64), torch.rand(5, 6))


def test_tiled_topk_aggregate_rejects_non_matrix_inputs():
    with pytest.raises(ValueError, match="rank-2"):
        tiled_topk_aggregate(torch.rand(2, 3, 4), torch.zeros(2, 3, 4, dtype=torch.int64), torch.rand(5, 6))


def test_tiled_topk_aggregate_requires_cuda():
    with pytest.raises(ValueError, match="requires CUDA"):
        tiled_topk_aggregate(torch.rand(2, 3), torch.zeros(2, 3, dtype=torch.int64), torch.rand(5, 6))


@pytest.mark.parametrize(
    ("q", "keys", "values", "gates", "k", "error", "message"),
    [
        (torch.rand(2, 3, 4), torch.rand(2, 5, 4), torch.rand(2, 5, 6), torch.rand(2, 3, 3), 2, ValueError,
         r"expected gates of shape \(2, 3, 2\)"),
        (torch.rand(2, 3, 4), torch.rand(2, 5, 3), torch.rand(2, 5, 6), None, 2, ValueError, "feature sizes must match"),
        (torch.rand(3, 4), torch.rand(2, 5, 4), torch.rand(2, 5, 6), None, 2, ValueError, "expected queries"),
        (torch.rand(2, 3, 4), torch.rand(2, 5, 4), torch.rand(2, 4, 6), None, 2, ValueError, "values must be"),
        (torch.rand(2, 3, 4), torch.rand(2, 5, 4), torch.rand(2, 5, 6), None, 11, ValueError, "top_k must be"),
        (torch.rand(2, 3, 4), torch.rand(2, 5, 4), torch.rand(2, 5, 6), None, 2, ValueError, "one CUDA device"),
        ([1.0], torch.rand(2, 5, 4), torch.rand(2, 5, 6), None, 2, TypeError, "queries must be a torch.Tensor"),
    ],
)
def test_gated_mixture_rejects_invalid_arguments(q, keys, values, gates, k, error, message):
    from sparsedict_b200 import gated_mixture_attention

    with pytest.raises(error, match=message):
        gated_mixture_attention(q, keys, values, k, gates)


def test_selection_operators_check_arguments():
    # messages of models/modules/topk_select.py:94-173 (SparseDict)
    from sparsedict_b200 import selection

    with pytest.raises(ValueError, match="selection must be 'hard' or 'ste'"):
        selection.sparse_topk_attention(torch.rand(3, 5), torch.rand(5, 2), 2, selection="soft")
    with pytest.raises(ValueError, match="expected scores with query and atom dimensions"):
        selection.straight_through_topk(torch.rand(5), 2)
    with pytest.raises(ValueError, match="floating-point dtype"):
        selection.hard_topk_mask(torch.ones(3, 5, dtype=torch.int64), 2)
    with pytest.raises(ValueError, match=r"k must be between 1 and 5; got 6"):
        selection.straight_through_topk(torch.rand(3, 5), 6)
    with pytest.raises(ValueError, match="CUDA"):
        selection.gumbel_perturbed_topk(torch.rand(3, 5), 2)


@pytest.mark.parametrize("kq,error,message", [
    ([[[1, 2, 3]]], TypeError, "k_per_query must be a torch.Tensor"),
    (torch.ones(1, 1, 3), ValueError, "integer dtype"),
    (torch.ones(1, 1, 4, dtype=torch.int32), ValueError, "must have shape"),
    (torch.zeros(1, 1, 3, dtype=torch.int32), ValueError, r"values must lie in \[1, 2\]"),
])
def test_adaptive_topk_rejects_invalid_budgets(kq, error, message):
    from sparsedict_b200 import adaptive_topk_attention

    q, k, v = torch.randn(1, 1, 3, 4), torch.randn(1, 1, 5, 4), torch.randn(1, 1, 5, 4)
    with pytest.raises(error, match=message):
        adaptive_topk_attention(q, k, v, kq, k_max=2)


def test_adaptive_topk_requires_cuda():
    from sparsedict_b200 import adaptive_topk_attention

    q, k, v = torch.randn(1, 1, 3, 4), torch.randn(1, 1, 5, 4), torch.randn(1, 1, 5, 4)
    with pytest.raises(ValueError, match="CUDA"):
        adaptive_topk_attention(q, k, v, torch.ones(1, 1, 3, dtype=torch.int32))
