"""Pins the CPU oracle against the reference's own outputs (golden vectors).

These run on CPU only.  The golden vectors were produced by the reference's
``sparse_topk_attention`` and ``torch.topk`` (``tests/golden/make_golden.py``).
"""

import itertools
import math

import numpy as np
import pytest

import oracle


def _flat(x):
    return x.reshape(-1, *x.shape[-2:])


def test_known_answer_indices(golden):
    vals, idx = oracle.topk_order(golden["known_scores"], 2)
    assert np.array_equal(idx, golden["known_indices"])
    assert np.array_equal(idx, [[1, 3], [0, 2]])


def test_configuration_1_forward_and_backward(golden):
    g = {k[5:]: v for k, v in golden.items() if k.startswith("cfg1_")}
    q, k, v, do = (_flat(g[n]) for n in ("q", "k", "v", "do"))
    scale = oracle.score_scale(q.shape[-1])
    out, idx, lse, _ = oracle.topk_attention_forward(q, k, v, 8, scale)
    assert np.array_equal(idx, _flat(g["idx"]))
    np.testing.assert_allclose(out, _flat(g["out"]), atol=1e-5, rtol=0)
    dq, dk, dv = oracle.topk_attention_backward(q, k, v, idx, do, scale)
    np.testing.assert_allclose(dq, _flat(g["dq"]), atol=1e-4, rtol=1e-3)
    np.testing.assert_allclose(dk, _flat(g["dk"]), atol=1e-4, rtol=1e-3)
    np.testing.assert_allclose(dv, _flat(g["dv"]), atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("grid", [(1, 13, 1, 24), (7, 64, 5, 67), (65, 129, 17, 33), (3, 73, 73, 7)])
def test_forward_parity_grids(golden, grid):
    tag = "grid_%d_%d_%d_%d" % grid
    q, k, v = (_flat(golden[f"{tag}_{n}"]) for n in "qkv")
    out, idx, _, _ = oracle.topk_attention_forward(q, k, v, grid[2], oracle.score_scale(64))
    assert np.array_equal(idx, _flat(golden[f"{tag}_idx"]))
    np.testing.assert_allclose(out, _flat(golden[f"{tag}_out"]), atol=1e-5, rtol=0)


def test_forward_parity_large_grid(golden):
    torch = pytest.importorskip("torch")
    torch.manual_seed(1234)
    q = torch.randn(1, 1, 4096, 64).numpy()
    k = torch.randn(1, 1, 256, 64).numpy()
    v = torch.randn(1, 1, 256, 64).numpy()
    tag = "grid_4096_256_16_64"
    chk = sum(np.float64(np.abs(a).sum()) for a in (q, k, v))
    assert chk == pytest.approx(float(golden[f"{tag}_checksum"]), rel=1e-12)
    out, idx, _, _ = oracle.topk_attention_forward(_flat(q), _flat(k), _flat(v), 16, oracle.score_scale(64))
    assert np.array_equal(idx, _flat(golden[f"{tag}_idx"]).astype(np.int32))
    np.testing.assert_allclose(out[:, ::8], _flat(golden[f"{tag}_out_rows8"]), atol=1e-5, rtol=0)


def test_float64_forward(golden):
    q, k, v = (_flat(golden[f"f64fwd_{n}"]) for n in "qkv")
    out, idx, lse, _ = oracle.topk_attention_forward(q, k, v, 5, oracle.score_scale(8))
    assert out.dtype == np.float64
    assert np.array_equal(idx, _flat(golden["f64fwd_idx"]))
    np.testing.assert_allclose(out, _flat(golden["f64fwd_out"]), atol=1e-12, rtol=0)


def test_float64_backward_matches_reference_autograd(golden):
    g = {k[7:]: v for k, v in golden.items() if k.startswith("f64bwd_")}
    q, k, v, do = (_flat(g[n]) for n in ("q", "k", "v", "do"))
    scale = oracle.score_scale(8)
    out, idx, _, _ = oracle.topk_attention_forward(q, k, v, 7, scale)
    assert np.array_equal(idx, _flat(g["idx"]))
    np.testing.assert_allclose(out, _flat(g["out"]), atol=1e-12, rtol=0)
    dq, dk, dv = oracle.topk_attention_backward(q, k, v, idx, do, scale)
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, _flat(g[name]), atol=1e-12, rtol=0)


@pytest.mark.parametrize("shape", [(1, 1, 7, 129, 8, 5, 7), (2, 2, 5, 263, 16, 33, 11)])
def test_hybrid_grids(golden, shape):
    tag = "hyb_" + "_".join(map(str, shape))
    q, k, v = (_flat(golden[f"{tag}_{n}"]) for n in "qkv")
    out, idx, _, _ = oracle.topk_attention_forward(q, k, v, shape[-1], oracle.score_scale(shape[4]))
    assert np.array_equal(idx, _flat(golden[f"{tag}_idx"]))
    np.testing.assert_allclose(out, _flat(golden[f"{tag}_out"]), atol=1e-5, rtol=0)


def test_hybrid_autograd(golden):
    g = {k[8:]: v for k, v in golden.items() if k.startswith("hybgrad_")}
    q, k, v, do = (_flat(g[n]) for n in ("q", "k", "v", "do"))
    scale = oracle.score_scale(8)
    out, idx, _, _ = oracle.topk_attention_forward(q, k, v, 5, scale)
    np.testing.assert_allclose(out, _flat(g["out"]), atol=1e-5, rtol=0)
    dq, dk, dv = oracle.topk_attention_backward(q, k, v, idx, do, scale)
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, _flat(g[name]), atol=1e-4, rtol=0)


@pytest.mark.parametrize("case", [(1, 1, 1), (7, 64, 5), (65, 129, 17), (8, 256, 64), (3, 73, 73)])
def test_topk_order_matches_torch_topk(golden, case):
    tag = "topk_%d_%d_%d" % case
    vals, idx = oracle.topk_order(golden[f"{tag}_scores"], case[2])
    assert np.array_equal(idx, golden[f"{tag}_idx"])
    assert np.array_equal(vals, golden[f"{tag}_vals"])


@pytest.mark.parametrize("case", [(1, 13, 1, 24), (7, 64, 5, 67), (65, 129, 17, 33), (3, 73, 73, 7)])
def test_aggregate_grids(golden, case):
    tag = "agg_%d_%d_%d_%d" % case
    ts, ti, vals = golden[f"{tag}_ts"], golden[f"{tag}_ti"], golden[f"{tag}_values"]
    w = np.exp(ts - ts.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    out = np.einsum("nk,nkf->nf", w, vals[ti])
    np.testing.assert_allclose(out, golden[f"{tag}_out"], atol=1e-5, rtol=0)
    sel_vals, sel_idx = oracle.topk_order(golden[f"{tag}_scores"], case[2])
    assert np.array_equal(sel_idx, ti)


def test_moe_routing_matches_reference_gate_fold(golden):
    g = {k[4:]: v for k, v in golden.items() if k.startswith("moe_")}
    experts = oracle.moe_route_top1(g["logits"])
    m = g["atoms"].shape[1]
    out, idx, _ = oracle.moe_topk_attention_forward(g["q"], g["atoms"], experts, 8, 1.0)
    assert np.array_equal(experts[:, None] * m + idx, g["flat_idx"])
    np.testing.assert_allclose(out, g["out"], atol=1e-5, rtol=0)
    dq, ddict = oracle.moe_topk_attention_backward(g["q"], g["atoms"], experts, idx, g["do"], 1.0)
    np.testing.assert_allclose(dq, g["dq"], atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(ddict, g["datoms"], atol=1e-5, rtol=1e-4)


def test_dense_reference_port_matches_sparse_oracle(golden):
    g = {k[5:]: v for k, v in golden.items() if k.startswith("cfg1_")}
    q, k, v, do = (_flat(g[n]) for n in ("q", "k", "v", "do"))
    scale = oracle.score_scale(q.shape[-1])
    out, idx, dq, dk, dv = oracle.dense_reference_fwd_bwd(q, k, v, do, 8, scale)
    np.testing.assert_allclose(out, _flat(g["out"]), atol=1e-5, rtol=0)
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, _flat(g[name]), atol=1e-4, rtol=1e-3)


def test_tie_rule_lower_index_first_brute_force():
    rng = np.random.default_rng(5)
    scores = rng.integers(-3, 4, size=(40, 23)).astype(np.float32)
    scores[3, 5] = np.nan
    scores[7, [1, 9]] = np.nan
    scores[11, :] = -np.inf
    for k in (1, 4, 23):
        vals, idx = oracle.topk_order(scores, k)
        for r in range(scores.shape[0]):
            def rank(j):
                s = scores[r, j]
                return (0 if np.isnan(s) else 1, 0.0 if np.isnan(s) else -float(s), j)
            expected = sorted(range(scores.shape[1]), key=rank)[:k]
            assert idx[r].tolist() == expected


def test_grid_quantisation_is_order_independent():
    rng = np.random.default_rng(9)
    d = 128
    q = np.clip(np.round(rng.standard_normal((1, 64, d)) * 8) / 8, -4, 4).astype(np.float32)
    k = np.clip(np.round(rng.standard_normal((1, 96, d)) * 8) / 8, -4, 4).astype(np.float32)
    s1 = oracle.quantize_to_grid(q, k, d, 64)
    perm = rng.permutation(d)
    s2 = oracle.quantize_to_grid(q[..., perm], k[..., perm], d, 64)
    assert np.array_equal(s1, s2)
    dots = np.einsum("bnd,bmd->bnm", q.astype(np.float64), k.astype(np.float64))
    exact = np.rint(np.float32(dots * 64) / np.float32(math.sqrt(d))) / 64
    assert np.array_equal(s1, exact.astype(np.float32))
    # many exact ties at the selection boundary
    _, idx = oracle.topk_order(s1, 8)
    assert idx.shape == (1, 64, 8)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf], dtype=np.float32)
    r = oracle.round_to_bf16(x)
    torch = pytest.importorskip("torch")
    expected = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(r, expected)
    rng = np.random.default_rng(0)
    y = rng.standard_normal(10000).astype(np.float32) * 7
    assert np.array_equal(oracle.round_to_bf16(y), torch.from_numpy(y).to(torch.bfloat16).float().numpy())


def test_gap_aware_mismatch_counter():
    scores = np.array([[5.0, 4.0, 3.99999, 1.0]], dtype=np.float32)
    assert oracle.gap_aware_index_mismatches(np.array([[0, 2]]), np.array([[0, 1]]), scores, 1e-4) == 0
    assert oracle.gap_aware_index_mismatches(np.array([[0, 3]]), np.array([[0, 1]]), scores, 1e-4) == 1
    # the near-tie allowance is reported: (failing rows, rows passing as near-ties)
    assert oracle.index_mismatch_counts(np.array([[0, 2]]), np.array([[0, 1]]), scores, 1e-4) == (0, 1)
    assert oracle.index_mismatch_counts(np.array([[0, 1]]), np.array([[0, 1]]), scores, 1e-4) == (0, 0)
    assert oracle.index_mismatch_counts(np.array([[2, 0]]), np.array([[0, 1]]), scores, 1e-4, ordered=False) == (0, 1)


def test_partition_top_k_matches_lexsort_order():
    from oracle.topk_attention import _topk_order_partition

    rng = np.random.default_rng(12)
    for dist in ("ints", "floats"):
        x = rng.integers(-4, 5, size=(30, 300)).astype(np.float32) if dist == "ints" else \
            rng.standard_normal((30, 300)).astype(np.float32)
        x[4, :50] = -np.inf
        for k in (1, 7, 64, 299, 300):
            v1, i1 = _topk_order_partition(x, k, x.shape)
            nan, value = np.isnan(x), x
            order = np.lexsort((np.broadcast_to(np.arange(300), x.shape), -value.astype(np.float64), ~nan), axis=-1)
            assert np.array_equal(i1, order[:, :k])


def test_unordered_set_comparison():
    scores = np.array([[5.0, 4.0, 3.99999, 1.0]], dtype=np.float32)
    assert oracle.gap_aware_index_mismatches(np.array([[1, 0]]), np.array([[0, 1]]), scores, 1e-4, ordered=False) == 0
    assert oracle.gap_aware_index_mismatches(np.array([[2, 0]]), np.array([[0, 1]]), scores, 1e-4, ordered=False) == 0
    assert oracle.gap_aware_index_mismatches(np.array([[3, 0]]), np.array([[0, 1]]), scores, 1e-4, ordered=False) == 1
    assert oracle.gap_aware_index_mismatches(np.array([[1, 0]]), np.array([[0, 1]]), scores, 1e-4, ordered=True) == 1


def test_gated_mixture_matches_reference_mixture(golden):
    # DualDomainMoEDictionary._mixture with soft gates (top-2 and dense
    # softmax rows, exact zeros), separate key and value projections
    g = {k[4:]: v for k, v in golden.items() if k.startswith("mix_")}
    out, idx, _, _ = oracle.gated_mixture_forward(g["q"], g["keys"], g["values"], g["gates"], 9)
    assert np.array_equal(idx, g["flat_idx"])
    np.testing.assert_allclose(out, g["out"], atol=1e-5, rtol=0)
    dq, dk, dv, dg = oracle.gated_mixture_backward(g["q"], g["keys"], g["values"], g["gates"], idx, g["do"])
    for got, name in ((dq, "dq"), (dk, "dkeys"), (dv, "dvalues"), (dg, "dgates")):
        np.testing.assert_allclose(got, g[name], atol=1e-5, rtol=1e-4)


def test_gate_bias_masks_zero_gates_and_clamps_tiny():
    gates = np.array([[0.0, 1e-45, 0.25, 1.0]], dtype=np.float32)
    bias = oracle.gate_bias(gates)
    assert bias[0, 0] == -np.inf
    assert bias[0, 1] == np.float32(np.log(np.finfo(np.float32).tiny))
    np.testing.assert_allclose(bias[0, 2:], np.log([0.25, 1.0]), rtol=1e-6)
