"""GPU parity of the CUDA path against the reference's golden vectors and the
CPU oracle.  Mirrors the reference's own GPU tests
(tests/test_triton_autograd.py, tests/test_hybrid_topk.py,
tests/test_fused_topk_attn.py) and adds bf16, tie-stress, routed and
full-size sampled-row cases.

Tolerances: fp32 outputs atol 1e-5 (reference pins) and gradients atol 1e-4 /
rtol 1e-3; fp64 atol 1e-9; bf16 rtol 2e-2.  Indices are compared exactly; on
non-quantised fp32 data a difference is accepted only between keys whose
oracle scores lie within 1e-5 of the k-th selected score (two summation
orders can swap a true near-tie).
"""

import math

import numpy as np
import pytest
import torch

import oracle
from sparsedict_b200 import (
    FusedTopKAttentionFunction,
    _native,
    _ops,
    fused_topk_attention,
    hybrid_topk_attention,
    tiled_affinity,
    tiled_topk,
    tiled_topk_aggregate,
)
from sparsedict_b200.kernels.hybrid_topk import _hybrid_topk_attention_with_aux
from sparsedict_b200.routed import routed_dictionary_attention

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _t(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    return t.to(dtype) if dtype is not None else t


def _flat(x):
    return x.reshape(-1, *x.shape[-2:])


def _oracle_scores64(q, k, scale):
    return np.einsum("bnd,bmd->bnm", _flat(q).astype(np.float64), _flat(k).astype(np.float64)) * scale


def _assert_indices(actual, expected, scores, tol=1e-5, ordered=True, max_near_ties=0):
    """Indices equal to the oracle's; a row may differ only by keys within ``tol``
    of the oracle's k-th score, and at most ``max_near_ties`` rows may do so
    (0 on the reference's golden grids)."""
    bad, near = oracle.index_mismatch_counts(actual, expected, scores, tol, ordered)
    assert bad == 0, f"{bad} rows select different keys"
    assert near <= max_near_ties, f"{near} rows differ inside the near-tie tolerance {tol} (limit {max_near_ties})"
    return near


# --- compile smoke -----------------------------------------------------------


def test_compile_smoke_fp32():
    torch.manual_seed(1234)
    q = torch.randn(1, 1, 512, 32, device=DEV)
    k = torch.randn(1, 1, 256, 32, device=DEV)
    v = torch.randn(1, 1, 256, 24, device=DEV)
    out = fused_topk_attention(q, k, v, 16)
    assert out.shape == (1, 1, 512, 24)
    assert torch.isfinite(out).all()


# --- forward parity against the reference's outputs --------------------------


@pytest.mark.parametrize("grid", [(1, 13, 1, 24), (7, 64, 5, 67), (65, 129, 17, 33), (3, 73, 73, 7)])
def test_forward_parity_fp32(golden, grid):
    tag = "grid_%d_%d_%d_%d" % grid
    q, k, v = (golden[f"{tag}_{n}"] for n in "qkv")
    out = fused_topk_attention(_t(q), _t(k), _t(v), grid[2])
    np.testing.assert_allclose(out.cpu().numpy(), golden[f"{tag}_out"], atol=1e-5, rtol=0)


def test_forward_parity_fp32_large_grid(golden):
    torch.manual_seed(1234)
    q = torch.randn(1, 1, 4096, 64)
    k = torch.randn(1, 1, 256, 64)
    v = torch.randn(1, 1, 256, 64)
    out = fused_topk_attention(q.to(DEV), k.to(DEV), v.to(DEV), 16)
    tag = "grid_4096_256_16_64"
    np.testing.assert_allclose(out.cpu().numpy()[..., ::8, :], golden[f"{tag}_out_rows8"], atol=1e-5, rtol=0)
    _, idx, _, _ = _hybrid_topk_attention_with_aux(q.to(DEV), k.to(DEV), v.to(DEV), 16, 1 / 8)
    # the reference's golden grid: no near-tie allowance used
    _assert_indices(idx.cpu().numpy(), _flat(golden[f"{tag}_idx"]), _oracle_scores64(q.numpy(), k.numpy(), 1 / 8))


def test_forward_parity_fp64(golden):
    q, k, v = (_t(golden[f"f64fwd_{n}"]) for n in "qkv")
    out = fused_topk_attention(q, k, v, 5)
    assert out.dtype == torch.float64
    np.testing.assert_allclose(out.cpu().numpy(), golden["f64fwd_out"], atol=1e-9, rtol=0)


def test_configuration_1_forward_backward(golden):
    g = {k[5:]: v for k, v in golden.items() if k.startswith("cfg1_")}
    q, k, v = (_t(g[n]).requires_grad_(True) for n in "qkv")
    out = fused_topk_attention(q, k, v, 8)
    np.testing.assert_allclose(out.detach().cpu().numpy(), g["out"], atol=1e-5, rtol=0)
    dq, dk, dv = torch.autograd.grad((out * _t(g["do"])).sum(), (q, k, v))
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got.cpu().numpy(), g[name], atol=1e-4, rtol=1e-3)
    scale = 1 / math.sqrt(32)
    _, idx, _, _ = _hybrid_topk_attention_with_aux(q.detach(), k.detach(), v.detach(), 8, scale)
    _assert_indices(idx.cpu().numpy(), _flat(g["idx"]), _oracle_scores64(g["q"], g["k"], scale))


# --- gradients ---------------------------------------------------------------


@pytest.mark.parametrize(("n", "m", "k", "dk", "dv"), [(8, 12, 5, 4, 3), (16, 32, 8, 8, 8)])
def test_gradcheck_fp64(n, m, k, dk, dv):
    torch.manual_seed(7)
    q = torch.randn(1, 1, n, dk, dtype=torch.float64, device=DEV, requires_grad=True)
    kk = torch.randn(1, 1, m, dk, dtype=torch.float64, device=DEV, requires_grad=True)
    v = torch.randn(1, 1, m, dv, dtype=torch.float64, device=DEV, requires_grad=True)
    torch.autograd.gradcheck(fused_topk_attention, (q, kk, v, k), eps=1e-6, atol=1e-4, nondet_tol=1e-5)


def test_forward_saves_inputs_support_indices_and_lse_only():
    torch.manual_seed(1234)
    q = torch.randn(1, 1, 8, 4, dtype=torch.float64, device=DEV, requires_grad=True)
    k = torch.randn(1, 1, 12, 4, dtype=torch.float64, device=DEV, requires_grad=True)
    v = torch.randn(1, 1, 12, 3, dtype=torch.float64, device=DEV, requires_grad=True)
    saved = []

    def pack(t):
        saved.append((tuple(t.shape), t.dtype))
        return t

    with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
        fused_topk_attention(q, k, v, 5)
    assert saved == [
        ((1, 8, 4), torch.float64),
        ((1, 12, 4), torch.float64),
        ((1, 12, 3), torch.float64),
        ((1, 8, 5), torch.int32),
        ((1, 8), torch.float64),
    ]


def test_backward_matches_reference_autograd_fp64(golden):
    g = {k[7:]: v for k, v in golden.items() if k.startswith("f64bwd_")}
    q, k, v = (_t(g[n]).requires_grad_(True) for n in "qkv")
    out = fused_topk_attention(q, k, v, 7)
    grads = torch.autograd.grad((out * _t(g["do"])).sum(), (q, k, v))
    for got, name in zip(grads, ("dq", "dk", "dv")):
        err = np.abs(got.cpu().numpy() - g[name]).max()
        assert err < 1e-9, f"{name} max abs err {err}"


def test_dq_is_bitwise_deterministic():
    torch.manual_seed(11)
    q = torch.randn(2, 2, 300, 64, device=DEV, requires_grad=True)
    k = torch.randn(2, 2, 700, 64, device=DEV)
    v = torch.randn(2, 2, 700, 64, device=DEV)
    do = torch.randn(2, 2, 300, 64, device=DEV)
    g1 = torch.autograd.grad((fused_topk_attention(q, k, v, 16) * do).sum(), q)[0]
    g2 = torch.autograd.grad((fused_topk_attention(q, k, v, 16) * do).sum(), q)[0]
    assert torch.equal(g1, g2)


# --- edge cases ---------------------------------------------------------------


def _oracle_out(q, k, v, topk, temperature=1.0):
    scale = oracle.score_scale(q.shape[-1], temperature)
    o, idx, lse, _ = oracle.topk_attention_forward(_flat(q), _flat(k), _flat(v), topk, scale)
    return o.reshape(*q.shape[:-1], v.shape[-1]), idx


def test_full_width_k_equals_m_fp32():
    torch.manual_seed(1234)
    q, k, v = torch.randn(1, 1, 32, 8), torch.randn(1, 1, 32, 8), torch.randn(1, 1, 32, 5)
    out = fused_topk_attention(q.to(DEV), k.to(DEV), v.to(DEV), 32)
    expected, _ = _oracle_out(q.numpy(), k.numpy(), v.numpy(), 32)
    np.testing.assert_allclose(out.cpu().numpy(), expected, atol=1e-5, rtol=0)


def test_single_key_for_64_dimensional_head():
    torch.manual_seed(1234)
    q, k, v = torch.randn(1, 1, 64, 64), torch.randn(1, 1, 1, 64), torch.randn(1, 1, 1, 3)
    out = fused_topk_attention(q.to(DEV), k.to(DEV), v.to(DEV), 1)
    expected, _ = _oracle_out(q.numpy(), k.numpy(), v.numpy(), 1)
    np.testing.assert_allclose(out.cpu().numpy(), expected, atol=1e-5, rtol=0)


def test_padded_candidates_zero_mass():
    torch.manual_seed(1234)
    q, k, v = (torch.randn(1, 1, 8, 4, device=DEV), torch.randn(1, 1, 5, 4, device=DEV),
               torch.randn(1, 1, 5, 4, device=DEV))
    assert torch.isfinite(fused_topk_attention(q, k, v, 2)).all()


@pytest.mark.parametrize("temperature", [0.5, 2.0])
def test_temperature_scales_scores(temperature):
    torch.manual_seed(3)
    q, k, v = torch.randn(2, 1, 50, 16), torch.randn(2, 1, 90, 16), torch.randn(2, 1, 90, 8)
    out = fused_topk_attention(q.to(DEV), k.to(DEV), v.to(DEV), 7, temperature)
    expected, _ = _oracle_out(q.numpy(), k.numpy(), v.numpy(), 7, temperature)
    np.testing.assert_allclose(out.cpu().numpy(), expected, atol=1e-5, rtol=0)


def test_ties_and_minus_inf_rows_follow_the_reference_order():
    # exact ties everywhere: integer-valued keys and a one-hot query
    q = torch.zeros(1, 1, 4, 4)
    q[..., 0] = 1.0
    k = torch.tensor([[3.0, 1, 3, 2, 3, 0, 2, 3, 1]]).T.repeat(1, 4).reshape(1, 1, 9, 4)
    v = torch.arange(9 * 2, dtype=torch.float32).reshape(1, 1, 9, 2)
    _, idx, _, _ = _hybrid_topk_attention_with_aux(q.to(DEV), k.to(DEV), v.to(DEV), 5, 1.0)
    assert idx[0, 0].tolist() == [0, 2, 4, 7, 3]


def _merging_temperature(hi, lo):
    """A temperature whose fp32 scale 1/(8T) (d = 64) is not a power of two and
    rounds the scores ``hi`` > ``lo`` to one fp32 value."""
    for t in np.linspace(0.55, 1.45, 9001):
        s = np.float32(1.0 / (float(t) * 8.0))
        if math.frexp(float(s))[0] != 0.5 and hi * s == lo * s:
            return float(t)
    raise AssertionError("no temperature merges the two scores")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("topk", [1, 2])
def test_scores_tied_by_the_scale_pick_the_lower_index(dtype, topk):
    # key 3 scores 1.75 - 2^-23 and key 300 scores 1.75; the scale rounds both
    # to one fp32 value, so the reference's order (larger scaled score, lower
    # index on ties) keeps key 3, whose raw score lies below the tensor-core
    # filter's bf16 bound 1.75.  At k = 2 key 100 (score 3) takes the first slot.
    hi = np.float32(1.75)
    lo = np.nextafter(hi, np.float32(0))
    temperature = _merging_temperature(hi, lo)
    m, d = 512, 64
    q = torch.zeros(1, 1, 128, d)
    q[..., 0] = 1.0
    q[..., 1] = 2.0 ** -23
    k = torch.zeros(1, 1, m, d)
    k[0, 0, 300, 0] = 1.75
    k[0, 0, 3, 0] = 1.75
    k[0, 0, 3, 1] = -1.0
    if topk == 2:
        k[0, 0, 100, 0] = 3.0
    v = torch.arange(m * d, dtype=torch.float32).reshape(1, 1, m, d) / (m * d)
    scale = 1.0 / (temperature * math.sqrt(d))
    _, idx, _, ts = _ops.topk_attn_fwd(_flat(q).to(DEV, dtype), _flat(k).to(DEV, dtype), _flat(v).to(DEV, dtype),
                                       topk, scale, want_scores=True)
    # the tensor-core forward keeps its selections in candidate-list order
    expected = [3] if topk == 1 else [3, 100]
    assert all(sorted(row) == expected for row in idx.tolist())
    assert (ts[idx == 3] == float(hi * np.float32(scale))).all()


# --- hybrid ------------------------------------------------------------------


@pytest.mark.parametrize("shape", [(1, 1, 7, 129, 8, 5, 7), (2, 2, 5, 263, 16, 33, 11)])
def test_hybrid_forward_matches_reference(golden, shape):
    tag = "hyb_" + "_".join(map(str, shape))
    q, k, v = (_t(golden[f"{tag}_{n}"]) for n in "qkv")
    out = hybrid_topk_attention(q, k, v, shape[-1])
    assert out.shape == (shape[0], shape[1], shape[2], shape[5])
    np.testing.assert_allclose(out.cpu().numpy(), golden[f"{tag}_out"], atol=1e-5, rtol=0)


def test_hybrid_custom_autograd_matches_reference(golden):
    g = {k[8:]: v for k, v in golden.items() if k.startswith("hybgrad_")}
    q, k, v = (_t(g[n]).requires_grad_(True) for n in "qkv")
    out = fused_topk_attention(q, k, v, 5)
    grads = torch.autograd.grad((out * _t(g["do"])).sum(), (q, k, v))
    np.testing.assert_allclose(out.detach().cpu().numpy(), g["out"], atol=1e-5, rtol=0)
    for got, name in zip(grads, ("dq", "dk", "dv")):
        np.testing.assert_allclose(got.cpu().numpy(), g[name], atol=1e-4, rtol=0)


def test_hybrid_aux_layout_and_lse():
    torch.manual_seed(5)
    q, k, v = torch.randn(2, 3, 40, 16), torch.randn(2, 3, 200, 16), torch.randn(2, 3, 200, 12)
    ts, ti, lse, out = _hybrid_topk_attention_with_aux(q.to(DEV), k.to(DEV), v.to(DEV), 9, 0.25)
    assert ts.shape == (6, 40, 9) and ts.dtype == torch.float32
    assert ti.shape == (6, 40, 9) and ti.dtype == torch.int32
    assert lse.shape == (6, 40) and out.shape == (6, 40, 12)
    o, idx, l, s = oracle.topk_attention_forward(_flat(q.numpy()), _flat(k.numpy()), _flat(v.numpy()), 9, 0.25)
    np.testing.assert_allclose(ts.cpu().numpy(), s, atol=1e-5, rtol=0)
    np.testing.assert_allclose(lse.cpu().numpy(), l, atol=1e-5, rtol=0)
    np.testing.assert_allclose(out.cpu().numpy(), o, atol=1e-5, rtol=0)
    with pytest.raises(ValueError, match="hybrid selector requires"):
        _hybrid_topk_attention_with_aux(q.to(DEV), k.to(DEV), v.to(DEV), 200, 0.25)


# --- stage ops -----------------------------------------------------------------


def test_tiled_affinity_matches_torch_fp16():
    torch.manual_seed(0)
    q = torch.randn(67, 24, device=DEV, dtype=torch.float16)
    k = torch.randn(129, 24, device=DEV, dtype=torch.float16)
    out = tiled_affinity(q, k)
    assert out.shape == (67, 129)
    assert torch.allclose(out, q.float() @ k.float().T, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("n,m,d", [(300, 1000, 64), (129, 257, 100), (1000, 4100, 200), (37, 700, 64)])
def test_tiled_affinity_fp16_tensor_cores(n, m, d):
    # fp16 rows with d >= 64 take the tcgen05 kernel: 128 x 256 score tiles,
    # features past d and rows past the ends read as zero; the products of
    # fp16 values are exact in fp32, so only the summation order differs.
    g = torch.Generator().manual_seed(n + m + d)
    q = torch.randn(n, d, generator=g).to(torch.float16)
    k = torch.randn(m, d, generator=g).to(torch.float16)
    out = tiled_affinity(q.to(DEV), k.to(DEV))
    assert out.dtype == torch.float32 and out.shape == (n, m)
    ref = q.double() @ k.double().T
    np.testing.assert_allclose(out.cpu().double().numpy(), ref.numpy(), atol=1e-4, rtol=1e-5)
    assert _native.device_status(clear=True) == 0


def test_tiled_affinity_fp16_strided_rows_both_kernels():
    # row strides of 104 halves (16-byte rows: tensor cores) and 100 halves
    # (the CUDA-core kernel) give the same scores
    torch.manual_seed(5)
    qb = torch.randn(260, 104, device=DEV, dtype=torch.float16)
    kb = torch.randn(300, 100, device=DEV, dtype=torch.float16)
    q, k = qb[:, :96], kb[:, :96]
    ref = q.double() @ k.double().T
    out = tiled_affinity(q, k)
    np.testing.assert_allclose(out.cpu().double().numpy(), ref.cpu().numpy(), atol=1e-4, rtol=1e-5)
    out2 = tiled_affinity(q, k.contiguous())
    np.testing.assert_allclose(out2.cpu().double().numpy(), ref.cpu().numpy(), atol=1e-4, rtol=1e-5)


def test_tiled_affinity_fp32_strided_rows():
    torch.manual_seed(1)
    base = torch.randn(70, 48, device=DEV)
    q = base[:, :40]
    k = torch.randn(130, 40, device=DEV)
    out = tiled_affinity(q, k)
    np.testing.assert_allclose(out.cpu().numpy(), q.cpu().double().numpy() @ k.cpu().double().numpy().T,
                               atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("case", [(1, 1, 1), (7, 64, 5), (65, 129, 17), (8, 256, 64), (3, 73, 73)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_tiled_topk_matches_torch_topk_indices(golden, case, dtype):
    tag = "topk_%d_%d_%d" % case
    vals, idx = tiled_topk(_t(golden[f"{tag}_scores"]).to(dtype), case[2])
    assert torch.equal(idx.cpu(), torch.from_numpy(golden[f"{tag}_idx"]))
    assert torch.equal(vals.cpu().float(), torch.from_numpy(golden[f"{tag}_vals"]))
    assert vals.dtype == dtype and idx.dtype == torch.int64


def test_tiled_topk_ties_and_nan_order():
    s = torch.tensor([[1.0, 3.0, 3.0, float("nan"), 2.0, 3.0, float("nan"), -float("inf")]], device=DEV)
    vals, idx = tiled_topk(s, 6)
    assert idx.tolist() == [[3, 6, 1, 2, 5, 4]]
    big = torch.randint(-2, 3, (40, 700), device=DEV).float()
    _, idx2 = tiled_topk(big, 65)
    _, exp_idx = oracle.topk_order(big.cpu().numpy(), 65)
    assert np.array_equal(idx2.cpu().numpy(), exp_idx)


@pytest.mark.parametrize("case", [(1, 13, 1, 24), (7, 64, 5, 67), (65, 129, 17, 33), (3, 73, 73, 7)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_tiled_topk_aggregate_matches_torch_reference(golden, case, dtype):
    tag = "agg_%d_%d_%d_%d" % case
    ts = _t(golden[f"{tag}_ts"]).to(dtype)
    ti = _t(golden[f"{tag}_ti"])
    vals = _t(golden[f"{tag}_values"]).to(dtype)
    out = tiled_topk_aggregate(ts, ti, vals)
    assert out.shape == (case[0], case[3]) and out.dtype == torch.float32
    w = torch.softmax(ts.float(), dim=1)
    expected = torch.sum(w.unsqueeze(-1) * vals.float()[ti], dim=1)
    assert (out - expected).abs().max().item() <= 1e-5
    if dtype == torch.float32:
        np.testing.assert_allclose(out.cpu().numpy(), golden[f"{tag}_out"], atol=1e-5, rtol=0)
    out32 = tiled_topk_aggregate(ts, ti.int(), vals)
    assert torch.equal(out, out32)


def test_aggregate_flags_out_of_range_indices():
    _native.device_status(clear=True)
    ts = torch.zeros(2, 3, device=DEV)
    ti = torch.tensor([[0, 1, 2], [0, 1, 9]], device=DEV)
    vals = torch.ones(4, 5, device=DEV)
    out = tiled_topk_aggregate(ts, ti, vals)
    assert _native.device_status(clear=True) & 1
    assert torch.allclose(out[0], torch.ones(5, device=DEV))
    assert torch.allclose(out[1], torch.full((5,), 2 / 3, device=DEV))


# --- bf16 / fp16 -------------------------------------------------------------------


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_low_precision_forward_backward_vs_oracle(dtype):
    torch.manual_seed(21)
    b, h, n, m, d, k = 2, 2, 384, 1000, 64, 32
    q, kk, v, do = (torch.randn(b, h, x, d) for x in (n, m, m, n))
    qd, kd, vd = (t.to(DEV, dtype).requires_grad_(True) for t in (q, kk, v))
    dod = do.to(DEV, dtype)
    out = fused_topk_attention(qd, kd, vd, k)
    assert out.dtype == dtype
    grads = torch.autograd.grad((out.float() * dod.float()).sum(), (qd, kd, vd))
    qr, kr, vr, dor = (t.detach().float().cpu().numpy() for t in (qd, kd, vd, dod))
    scale = 1 / 8
    o, idx, _, _ = oracle.topk_attention_forward(_flat(qr), _flat(kr), _flat(vr), k, scale)
    from sparsedict_b200 import _ops

    _, gidx, _, _ = _ops.topk_attn_fwd(*(t.detach().reshape(b * h, -1, d) for t in (qd, kd, vd)), k, scale)
    gidx = gidx.cpu().numpy().reshape(idx.shape)
    # selected sets agree wherever the affinity gap exceeds bf16 rounding (here: 1e-4);
    # the tensor-core kernel returns each row's top-k set unordered
    _assert_indices(gidx, idx, _oracle_scores64(qr, kr, scale), tol=1e-4, ordered=False, max_near_ties=2)
    np.testing.assert_allclose(out.float().detach().cpu().numpy().reshape(o.shape), o, rtol=2e-2, atol=2e-2)
    # backward checked on the support the GPU selected
    ref = oracle.topk_attention_backward(_flat(qr), _flat(kr), _flat(vr), gidx, _flat(dor), scale)
    for got, exp in zip(grads, ref):
        got = got.float().cpu().numpy().reshape(exp.shape)
        assert np.abs(got - exp).max() <= 2e-2 * max(1.0, np.abs(exp).max())


@pytest.mark.parametrize("n,m,k", [(300, 1000, 32), (512, 4096, 64), (100, 129, 1), (257, 2000, 7)])
def test_bf16_tensor_core_exact_ties_lower_index_wins(n, m, k):
    # Integer-valued bf16 queries and keys: every score is an exact integer
    # (no rounding anywhere), most of them tied.  Rows whose bucketed
    # candidate lists cannot be shrunk go through the exact warp
    # re-selection; either way the selected set must be the oracle's, with
    # the lower key index winning every tie.
    g = torch.Generator().manual_seed(n + m + k)
    bh, d = 3, 64
    q, kk = (torch.randint(-2, 3, (bh, x, d), generator=g).to(torch.bfloat16) for x in (n, m))
    v = torch.randn(bh, m, d, generator=g).to(torch.bfloat16)
    from sparsedict_b200 import _ops

    out, idx, lse, _ = _ops.topk_attn_fwd(q.to(DEV), kk.to(DEV), v.to(DEV), k, 1 / 8)
    assert _native.device_status(clear=True) == 0
    qf, kf, vf = (t.float().numpy() for t in (q, kk, v))
    o, oi, ol, _ = oracle.topk_attention_forward(qf, kf, vf, k, 1 / 8)
    got = np.sort(idx.cpu().numpy().reshape(-1, k), axis=1)
    assert np.array_equal(got, np.sort(oi.reshape(-1, k), axis=1))
    np.testing.assert_allclose(lse.cpu().numpy().reshape(ol.shape), ol, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out.float().cpu().numpy(), o, rtol=2e-2, atol=2e-2)


def test_tensor_core_forward_on_caller_workspace_matches_library_pool():
    # The same forward through sdk_topk_attn_fwd (library memory pool) and
    # sdk_topk_attn_fwd_ws (a torch-allocated workspace) gives identical
    # results; a workspace one byte short, or misaligned, is refused before
    # anything is launched.
    lib = _native.load()
    g = torch.Generator().manual_seed(11)
    bh, n, m, d, k = 2, 300, 1000, 64, 16
    q, kk, v = (torch.randn(bh, x, d, generator=g).to(torch.bfloat16).to(DEV) for x in (n, m, m))
    stream = torch.cuda.current_stream().cuda_stream

    def run(ws, nbytes, pooled=False):
        out = torch.zeros(bh, n, d, device=DEV, dtype=torch.bfloat16)
        idx = torch.zeros(bh * n, k, device=DEV, dtype=torch.int32)
        lse = torch.zeros(bh * n, device=DEV)
        args = (q.data_ptr(), kk.data_ptr(), v.data_ptr(), out.data_ptr(), idx.data_ptr(), lse.data_ptr(),
                None, None, None, bh, n, m, d, d, k, 0.125, 0, _native.DTYPE_BF16)
        rc = lib.sdk_topk_attn_fwd(*args, stream) if pooled else lib.sdk_topk_attn_fwd_ws(*args, ws, nbytes, stream)
        torch.cuda.synchronize()
        return rc, out, idx, lse

    need = lib.sdk_topk_attn_fwd_workspace_size(bh * n, m, d, d, k, 0, 0, _native.DTYPE_BF16)
    assert need == bh * n * (192 * 2 + 20)
    buf = torch.empty(need + 16, device=DEV, dtype=torch.uint8)
    rc0, o0, i0, l0 = run(None, 0, pooled=True)
    rc1, o1, i1, l1 = run(buf.data_ptr(), need)
    assert rc0 == rc1 == _native.SDK_OK
    assert torch.equal(o0, o1) and torch.equal(i0, i1) and torch.equal(l0, l1)
    assert run(buf.data_ptr(), need - 1)[0] == _native.SDK_ERR_INVALID_ARGUMENT
    assert run(buf.data_ptr() + 4, need)[0] == _native.SDK_ERR_INVALID_ARGUMENT
    assert _native.device_status(clear=True) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_forward_unsafe_inputs_are_reselected_exactly(dtype):
    # The fused stream filter assumes no score can overflow.  A query row
    # holding NaN, a query row holding inf and, for bf16, a key slice holding
    # a value of 2^100 fail the input check; those rows are re-selected
    # exactly and must follow the reference order (NaN scores first, lower
    # key index first on ties), the other rows take the fused path.
    g = torch.Generator().manual_seed(23)
    bh, n, m, d, k = 3, 300, 1000, 64, 16
    q, kk = (torch.randn(bh, x, d, generator=g) for x in (n, m))
    v = torch.randn(bh, m, d, generator=g)
    q[0, 5, 3] = float("nan")
    q[2, 7, 9] = float("inf")
    if dtype == torch.bfloat16:
        kk[1, 17, 0] = 2.0 ** 100
    q, kk, v = (t.to(dtype) for t in (q, kk, v))
    from sparsedict_b200 import _ops

    out, idx, lse, _ = _ops.topk_attn_fwd(q.to(DEV), kk.to(DEV), v.to(DEV), k, 1 / 8)
    assert _native.device_status(clear=True) == 0
    got = idx.cpu().numpy().reshape(bh, n, k)
    qf, kf, vf = (t.double().numpy() for t in (q, kk, v))
    _, oi, _, _ = oracle.topk_attention_forward(qf, kf, vf, k, 1 / 8)
    # the NaN row: every score NaN, so keys 0..k-1
    assert sorted(got[0, 5]) == list(range(k))
    scores = _oracle_scores64(qf, kf, 1 / 8)
    finite = np.isfinite(scores).all(axis=-1)
    exp = np.sort(oi.reshape(bh, n, k), axis=-1)
    act = np.sort(got, axis=-1)
    assert np.array_equal(act[~finite], exp[~finite])
    _assert_indices(act[finite][None], exp[finite][None], scores[finite][None], tol=1e-4, ordered=False,
                    max_near_ties=2)
    if dtype == torch.bfloat16:
        # q·k of key 17 in slice 1 is about +-2^100·q[0]: first or excluded
        top = (qf[1, :, 0] > 0)
        assert (got[1][top] == 17).any(axis=-1).all()


# --- tie stress (configuration 5 shape family, reduced size) ----------------------


def _grid_inputs(seed, bh, n, m, d):
    rng = np.random.default_rng(seed)
    q = np.clip(np.round(rng.standard_normal((bh, n, d)) * 8) / 8, -4, 4).astype(np.float32)
    k = np.clip(np.round(rng.standard_normal((bh, m, d)) * 8) / 8, -4, 4).astype(np.float32)
    v = rng.standard_normal((bh, m, d)).astype(np.float32)
    do = rng.standard_normal((bh, n, d)).astype(np.float32)
    return q, k, v, do


@pytest.mark.parametrize("topk", [1, 128])
def test_tie_stress_grid_indices_bit_exact(topk):
    bh, n, m, d = 4, 512, 1024, 128
    q, k, v, do = _grid_inputs(17 + topk, bh, n, m, d)
    qd, kd, vd = (_t(x.reshape(1, bh, *x.shape[1:])).requires_grad_(True) for x in (q, k, v))
    out = FusedTopKAttentionFunction.apply(qd, kd, vd, topk, 1.0, 64)
    scores = oracle.quantize_to_grid(q, k, d, 64)
    _, exp_idx = oracle.topk_order(scores, topk)
    o, _, _, _ = oracle.topk_attention_forward(q, k, v, topk, 1 / math.sqrt(d), scores=scores)
    np.testing.assert_allclose(out.detach().cpu().numpy().reshape(o.shape), o, atol=1e-5, rtol=1e-5)
    grads = torch.autograd.grad((out * _t(do.reshape(1, bh, n, d))).sum(), (qd, kd, vd))
    ref = oracle.topk_attention_backward(q, k, v, exp_idx, do, 1 / math.sqrt(d), scores=scores)
    for got, exp in zip(grads, ref):
        np.testing.assert_allclose(got.cpu().numpy().reshape(exp.shape), exp, atol=1e-4, rtol=1e-3)
    # bit-exact indices through the forward with saved support
    from sparsedict_b200 import _ops

    _, idx, _, _ = _ops.topk_attn_fwd(_t(q), _t(k), _t(v), topk, 1 / math.sqrt(d), score_grid=64)
    assert np.array_equal(idx.cpu().numpy().reshape(exp_idx.shape), exp_idx)


# --- routed dictionaries (configuration 3 shape family, reduced size) -------------


def test_routed_dictionary_attention_matches_reference(golden):
    g = {k[4:]: v for k, v in golden.items() if k.startswith("moe_")}
    q = _t(g["q"]).requires_grad_(True)
    atoms = _t(g["atoms"]).requires_grad_(True)
    out, expert, _ = routed_dictionary_attention(q, atoms, _t(g["logits"]), 8, 1.0, return_routing=True)
    assert np.array_equal(expert.cpu().numpy(), oracle.moe_route_top1(g["logits"]))
    np.testing.assert_allclose(out.detach().cpu().numpy(), g["out"], atol=1e-5, rtol=0)
    dq, datoms = torch.autograd.grad((out * _t(g["do"])).sum(), (q, atoms))
    np.testing.assert_allclose(dq.cpu().numpy(), g["dq"], atol=1e-4, rtol=1e-3)
    np.testing.assert_allclose(datoms.cpu().numpy(), g["datoms"], atol=1e-4, rtol=1e-3)


def test_routed_bf16_full_configuration_sampled_rows():
    torch.manual_seed(3)
    n, d, e, m, k = 16384, 64, 8, 1024, 16
    q = torch.randn(n, d)
    atoms = torch.randn(e, m, d) / math.sqrt(d)
    logits = torch.randn(n, e)
    qd, ad = q.to(DEV, torch.bfloat16), atoms.to(DEV, torch.bfloat16)
    out = routed_dictionary_attention(qd, ad, logits.to(DEV), k, 1.0)
    rows = np.random.default_rng(0).choice(n, 256, replace=False)
    experts = oracle.moe_route_top1(logits.numpy())
    qr, ar = qd.float().cpu().numpy(), ad.float().cpu().numpy()
    o, _, _ = oracle.moe_topk_attention_forward(qr[rows], ar, experts[rows], k, 1.0)
    np.testing.assert_allclose(out.float().cpu().numpy()[rows], o, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize(("n", "e"), [(1, 1), (255, 3), (16384, 8), (70001, 16)])
def test_route_top1_is_a_stable_grouping(n, e):
    # expert = first maximum (NaN ranks highest, the lower expert on ties);
    # order = tokens grouped by expert in ascending token order; offsets.
    from sparsedict_b200 import _ops

    rng = np.random.default_rng(n + e)
    logits = rng.standard_normal((n, e)).astype(np.float32)
    logits[rng.random(n) < 0.05] = 0.5  # whole-row ties
    logits[rng.random((n, e)) < 0.01] = np.nan
    expert, order, offsets = _ops.route_top1(torch.from_numpy(logits).to(DEV))
    assert _native.device_status(clear=True) == 0
    exp = oracle.moe_route_top1(logits)
    assert np.array_equal(expert.cpu().numpy(), exp)
    assert np.array_equal(order.cpu().numpy(), np.argsort(exp, kind="stable"))
    assert np.array_equal(offsets.cpu().numpy(), np.concatenate([[0], np.cumsum(np.bincount(exp, minlength=e))]))


def _routed_case(sizes, m, k, seed):
    """Queries routed to experts with exactly ``sizes[e]`` tokens each (tokens shuffled)."""
    rng = np.random.default_rng(seed)
    e, n, d = len(sizes), int(sum(sizes)), 64
    experts = rng.permutation(np.repeat(np.arange(e), sizes))
    logits = rng.standard_normal((n, e)).astype(np.float32)
    logits[np.arange(n), experts] += 20.0
    q = oracle.round_to_bf16(rng.standard_normal((n, d)).astype(np.float32))
    atoms = oracle.round_to_bf16((rng.standard_normal((e, m, d)) / 8).astype(np.float32))
    return q, atoms, logits, experts


@pytest.mark.parametrize(("sizes", "m", "k"), [((0, 1, 255, 256, 257, 700), 320, 16),
                                               ((513, 0, 0, 40, 7, 1), 1024, 64),
                                               ((300,) * 8, 96, 1)])
def test_routed_tensor_core_ragged_experts(sizes, m, k):
    # Expert groups of 0, 1, just under / at / over one 256-row CTA and several
    # CTAs, and key counts that end in a partial 128-key tile: selected index
    # sets (grouped row order), outputs and LSE against the oracle, bf16 d=64
    # (the tensor-core forward).
    from sparsedict_b200 import _ops

    q, atoms, logits, experts = _routed_case(sizes, m, k, seed=sum(sizes) + m + k)
    qd = torch.from_numpy(q).to(DEV, torch.bfloat16)
    ad = torch.from_numpy(atoms).to(DEV, torch.bfloat16)
    out, expert, idx = routed_dictionary_attention(qd, ad, torch.from_numpy(logits).to(DEV), k, 1.0,
                                                   return_routing=True)
    assert _native.device_status(clear=True) == 0
    assert np.array_equal(expert.cpu().numpy(), experts)
    o, oidx, olse = oracle.moe_topk_attention_forward(q, atoms, experts, k, 1.0)
    order = np.argsort(experts, kind="stable")
    sc = np.stack([q[t].astype(np.float64) @ atoms[experts[t]].astype(np.float64).T for t in order])
    _assert_indices(idx.cpu().numpy()[None], oidx[order][None], sc[None], tol=1e-4, ordered=False,
                    max_near_ties=max(1, len(order) // 100))
    np.testing.assert_allclose(out.float().cpu().numpy(), o, rtol=2e-2, atol=2e-2)
    # the same call through the op: grouped LSE in the accumulator type
    _, order_d, offsets = _ops.route_top1(torch.from_numpy(logits).to(DEV))
    _, _, lse, _ = _ops.topk_attn_fwd(qd, ad, ad, k, 1.0, row_offsets=offsets, row_index=order_d)
    np.testing.assert_allclose(lse.cpu().numpy(), olse[order], rtol=1e-5, atol=1e-5)


def test_grouped_rows_without_permutation_tensor_core():
    # Grouped slices whose query rows are already in slice order (offsets, no
    # row index): the tensor-core forward reads them by TMA across slice ends.
    from sparsedict_b200 import _ops

    sizes, m, k = (130, 0, 383, 1, 256), 256, 32
    q, atoms, _, _ = _routed_case(sizes, m, k, seed=7)
    experts = np.repeat(np.arange(len(sizes)), sizes)
    qd = torch.from_numpy(q).to(DEV, torch.bfloat16)
    ad = torch.from_numpy(atoms).to(DEV, torch.bfloat16)
    offsets = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32, device=DEV)
    out, idx, lse, _ = _ops.topk_attn_fwd(qd, ad, ad, k, 1.0, row_offsets=offsets)
    assert _native.device_status(clear=True) == 0
    o, oidx, olse = oracle.moe_topk_attention_forward(q, atoms, experts, k, 1.0)
    sc = np.stack([q[t].astype(np.float64) @ atoms[experts[t]].astype(np.float64).T for t in range(len(q))])
    _assert_indices(idx.cpu().numpy()[None], oidx[None], sc[None], tol=1e-4, ordered=False,
                    max_near_ties=max(1, len(q) // 100))
    np.testing.assert_allclose(out.float().cpu().numpy(), o, rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(lse.cpu().numpy(), olse, rtol=1e-5, atol=1e-5)


def test_routed_bf16_full_configuration_index_sets():
    # Configuration 3 at full size (N=16384 tokens, E=8 experts of M=1024
    # atoms, k=16, bf16): every token's selected set against the oracle.
    torch.manual_seed(3)
    n, d, e, m, k = 16384, 64, 8, 1024, 16
    q = torch.randn(n, d).to(torch.bfloat16)
    atoms = (torch.randn(e, m, d) / math.sqrt(d)).to(torch.bfloat16)
    logits = torch.randn(n, e)
    out, expert, idx = routed_dictionary_attention(q.to(DEV), atoms.to(DEV), logits.to(DEV), k, 1.0,
                                                   return_routing=True)
    assert _native.device_status(clear=True) == 0
    qr, ar = q.float().numpy(), atoms.float().numpy()
    experts = oracle.moe_route_top1(logits.numpy())
    assert np.array_equal(expert.cpu().numpy(), experts)
    order = np.argsort(experts, kind="stable")
    gidx = idx.cpu().numpy()
    near = 0
    for ex in range(e):
        rows = order[experts[order] == ex]
        pos = np.nonzero(experts[order] == ex)[0]
        o, oidx, _, _ = oracle.topk_attention_forward(qr[rows][None], ar[ex][None], ar[ex][None], k, 1.0)
        sc = (qr[rows].astype(np.float64) @ ar[ex].astype(np.float64).T)[None]
        near += _assert_indices(gidx[pos][None], oidx, sc, tol=1e-4, ordered=False, max_near_ties=len(rows))
        np.testing.assert_allclose(out.float().cpu().numpy()[rows], o[0], rtol=2e-2, atol=2e-2)
    assert near <= max(1, n // 100), f"{near} near-tie rows"


# --- full-size configurations, sampled rows against the oracle --------------------


def _oracle_slice_backward(q, k, v, idx, do, scale, chunk=2048):
    """Float64 oracle gradients of one whole slice, in row chunks (dK/dV summed)."""
    dq = np.zeros(q.shape, np.float64)
    dk = np.zeros(k.shape, np.float64)
    dv = np.zeros(v.shape, np.float64)
    for r0 in range(0, q.shape[0], chunk):
        r1 = min(q.shape[0], r0 + chunk)
        a, b, c = oracle.topk_attention_backward(q[None, r0:r1], k[None], v[None], idx[None, r0:r1],
                                                 do[None, r0:r1], scale)
        dq[r0:r1] = a[0]
        dk += b[0]
        dv += c[0]
    return dq, dk, dv


@pytest.mark.parametrize(("b", "h", "n", "m", "d", "k"), [(8, 8, 4096, 4096, 64, 32), (16, 8, 16384, 16384, 64, 64)])
def test_full_size_bf16_index_sets_outputs_and_gradients(b, h, n, m, d, k):
    # The benchmarked shapes at full size (configuration 2: B=8 H=8 N=M=4096
    # k=32; configuration 4: B=16 H=8 N=M=16384 k=64), bf16.  For sampled rows
    # of four slices: the selected index SET equals the oracle's except where
    # the keys that differ score within 1e-4 of the oracle's k-th score (at
    # most 1 % of the rows may use that allowance), outputs and LSE, and dQ
    # on the GPU's support.  For one whole slice: dK and dV against the
    # float64 oracle.  The public API's output equals the op's bit for bit.
    gen = torch.Generator(device=DEV).manual_seed(2024)
    q = torch.randn(b, h, n, d, device=DEV, generator=gen).to(torch.bfloat16)
    kk = torch.randn(b, h, m, d, device=DEV, generator=gen).to(torch.bfloat16)
    v = torch.randn(b, h, m, d, device=DEV, generator=gen).to(torch.bfloat16)
    do = torch.randn(b, h, n, d, device=DEV, generator=gen).to(torch.bfloat16)
    scale = 1 / math.sqrt(d)
    from sparsedict_b200 import _ops

    s_all = b * h
    q3, k3, v3, do3 = (t.reshape(s_all, -1, d) for t in (q, kk, v, do))
    out, idx, lse, _ = _ops.topk_attn_fwd(q3, k3, v3, k, scale)
    assert torch.equal(fused_topk_attention(q, kk, v, k).reshape(out.shape), out)
    idx3, lse2 = idx.view(s_all, n, k), lse.view(s_all, n)
    dq, dk_acc, dv_acc = _ops.topk_attn_bwd(q3, k3, v3, do3, idx3, lse2, scale)
    assert _native.device_status(clear=True) == 0
    rng = np.random.default_rng(1)
    slices = rng.choice(s_all, 4, replace=False)
    rows = np.sort(rng.choice(n, 64, replace=False))
    near = 0
    for s in slices:
        qs, ks, vs, ds = (t[s].float().cpu().numpy() for t in (q3, k3, v3, do3))
        o, oidx, olse, _ = oracle.topk_attention_forward(qs[None, rows], ks[None], vs[None], k, scale)
        gidx = idx3[s, rows].cpu().numpy()
        sc = np.einsum("nd,md->nm", qs[rows].astype(np.float64), ks.astype(np.float64)) * scale
        near += _assert_indices(gidx[None], oidx, sc[None], tol=1e-4, ordered=False, max_near_ties=len(rows))
        np.testing.assert_allclose(out[s, rows].float().cpu().numpy(), o[0], rtol=2e-2, atol=2e-2)
        np.testing.assert_allclose(lse2[s, rows].cpu().numpy(), olse[0], rtol=1e-5, atol=1e-5)
        rdq, _, _ = oracle.topk_attention_backward(qs[None, rows], ks[None], vs[None], gidx[None], ds[None, rows],
                                                   scale)
        got = dq[s, rows].float().cpu().numpy()
        assert np.abs(got - rdq[0]).max() <= 2e-2 * max(1.0, np.abs(rdq).max())
    assert near <= max(1, len(slices) * len(rows) // 100), f"{near} near-tie rows"
    s0 = int(slices[0])
    qs, ks, vs, ds = (t[s0].float().cpu().numpy() for t in (q3, k3, v3, do3))
    _, rdk, rdv = _oracle_slice_backward(qs, ks, vs, idx3[s0].cpu().numpy(), ds, scale)
    for got, exp in ((dk_acc[s0], rdk), (dv_acc[s0], rdv)):
        np.testing.assert_allclose(got.float().cpu().numpy(), exp, rtol=1e-3, atol=1e-3 * np.abs(exp).max())


def test_routed_bf16_backward_vs_oracle():
    torch.manual_seed(4)
    n, d, e, m, k = 2048, 64, 4, 512, 16
    q = torch.randn(n, d)
    atoms = torch.randn(e, m, d) / 8
    logits = torch.randn(n, e)
    do = torch.randn(n, d)
    qd = q.to(DEV, torch.bfloat16).requires_grad_(True)
    ad = atoms.to(DEV, torch.bfloat16).requires_grad_(True)
    out = routed_dictionary_attention(qd, ad, logits.to(DEV), k, 1.0)
    dq, da = torch.autograd.grad((out.float() * do.to(DEV)).sum(), (qd, ad))
    qr, ar = qd.detach().float().cpu().numpy(), ad.detach().float().cpu().numpy()
    experts = oracle.moe_route_top1(logits.numpy())
    o, idx, _ = oracle.moe_topk_attention_forward(qr, ar, experts, k, 1.0)
    np.testing.assert_allclose(out.detach().float().cpu().numpy(), o, rtol=2e-2, atol=2e-2)
    gq, ga = oracle.moe_topk_attention_backward(qr, ar, experts, idx, do.numpy(), 1.0)
    for got, exp in ((dq, gq), (da, ga)):
        got = got.float().cpu().numpy()
        assert np.abs(got - exp).max() <= 2e-2 * max(1.0, np.abs(exp).max())


@pytest.mark.parametrize("topk", [1, 128])
def test_tie_stress_full_configuration_sampled_rows_bit_exact(topk):
    # B=4, H=4, N=M=8192, d=128, fp32; Q and K on a 1/8 grid clamped to [-4, 4] so every
    # dot product is exact; scores rounded to the 1/64 grid before selection (many exact
    # ties); the lower key index must win every tie.
    from sparsedict_b200 import _ops

    bh, n, m, d = 16, 8192, 8192, 128
    gen = torch.Generator(device=DEV).manual_seed(55 + topk)
    q = torch.clamp(torch.round(torch.randn(bh, n, d, device=DEV, generator=gen) * 8) / 8, -4, 4)
    k = torch.clamp(torch.round(torch.randn(bh, m, d, device=DEV, generator=gen) * 8) / 8, -4, 4)
    v = torch.randn(bh, m, d, device=DEV, generator=gen)
    out, idx, _, _ = _ops.topk_attn_fwd(q, k, v, topk, 1 / math.sqrt(d), score_grid=64)
    rng = np.random.default_rng(topk)
    for s in rng.choice(bh, 3, replace=False):
        rows = rng.choice(n, 64, replace=False)
        qs = q[s, rows].cpu().numpy()[None]
        ks = k[s].cpu().numpy()[None]
        scores = oracle.quantize_to_grid(qs, ks, d, 64)
        _, exp_idx = oracle.topk_order(scores, topk)
        got = idx.view(bh, n, topk)[s, rows].cpu().numpy()
        assert np.array_equal(got, exp_idx[0])
        o, _, _, _ = oracle.topk_attention_forward(qs, ks, v[s].cpu().numpy()[None], topk, 1 / math.sqrt(d),
                                                   scores=scores)
        np.testing.assert_allclose(out.view(bh, n, d)[s, rows].cpu().numpy(), o[0], atol=1e-5, rtol=1e-5)


# --- gated mixture (DualDomainMoEDictionary._mixture) -----------------------------


def test_gated_mixture_matches_reference_fp32(golden):
    from sparsedict_b200 import _ops, gated_mixture_attention

    g = {k[4:]: v for k, v in golden.items() if k.startswith("mix_")}
    q, keys, values, gates = (_t(g[n]).requires_grad_(True) for n in ("q", "keys", "values", "gates"))
    out = gated_mixture_attention(q, keys, values, 9, gates)
    np.testing.assert_allclose(out.detach().cpu().numpy(), g["out"], atol=1e-5, rtol=0)
    grads = torch.autograd.grad((out * _t(g["do"])).sum(), (q, keys, values, gates))
    for got, name in zip(grads, ("dq", "dkeys", "dvalues", "dgates")):
        np.testing.assert_allclose(got.cpu().numpy(), g[name], atol=1e-4, rtol=1e-3)
    # the selection itself: the biased forward picks the reference's flat indices
    b, n, dk = g["q"].shape
    e, m, _ = g["keys"].shape
    bias = torch.where(gates == 0, torch.full_like(gates, float("-inf")),
                       gates.clamp_min(torch.finfo(torch.float32).tiny).log()).detach().reshape(b * n, e)
    _, idx, _, _ = _ops.topk_attn_fwd(q.detach().reshape(1, b * n, dk), keys.detach().reshape(1, e * m, dk),
                                      values.detach().reshape(1, e * m, -1), 9, 1.0, seg_bias=bias.contiguous())
    assert np.array_equal(idx.cpu().numpy().reshape(b, n, 9), g["flat_idx"])


def test_gated_mixture_bf16_vs_oracle():
    from sparsedict_b200 import gated_mixture_attention

    gen = torch.Generator().manual_seed(17)
    b, n, dk, c, e, m, k = 2, 300, 64, 64, 8, 256, 16
    q = torch.randn(b, n, dk, generator=gen).to(torch.bfloat16)
    keys = (torch.randn(e, m, dk, generator=gen) / 8).to(torch.bfloat16)
    values = torch.randn(e, m, c, generator=gen).to(torch.bfloat16)
    logits = torch.randn(b, n, e, generator=gen)
    top_l, top_e = logits.topk(2, dim=-1)
    gates = torch.zeros_like(logits).scatter(-1, top_e, torch.softmax(top_l, -1)).to(torch.bfloat16)
    do = torch.randn(b, n, c, generator=gen).to(torch.bfloat16)
    qd, kd, vd, gd = (t.to(DEV).requires_grad_(True) for t in (q, keys, values, gates))
    out = gated_mixture_attention(qd, kd, vd, k, gd)
    grads = torch.autograd.grad((out.float() * do.to(DEV).float()).sum(), (qd, kd, vd, gd))
    qf, kf, vf, gf, dof = (t.float().numpy() for t in (q, keys, values, gates, do))
    o, idx, _, _ = oracle.gated_mixture_forward(qf, kf, vf, gf, k)
    np.testing.assert_allclose(out.float().detach().cpu().numpy(), o, rtol=2e-2, atol=2e-2)
    ref = oracle.gated_mixture_backward(qf, kf, vf, gf, idx, dof)
    for got, exp in zip(grads, ref):
        got = got.float().cpu().numpy()
        assert np.abs(got - exp).max() <= 2e-2 * max(1.0, np.abs(exp).max())


def test_gated_mixture_tensor_core_bias_rows():
    # bf16, d = 64 and whole 128-atom expert segments: the biased forward on
    # the tensor cores.  Top-2 gates (six experts at -inf per token), a token
    # whose gates are all 0 (every score -inf: the k lowest indices, NaN
    # output), one with a NaN gate (NaN scores rank first) and one with a gate
    # below the clamp.  Flat index sets against the oracle (near ties aside),
    # outputs and LSE.
    from sparsedict_b200 import _ops

    gen = torch.Generator().manual_seed(23)
    b, n, dk, e, m, k = 1, 700, 64, 8, 128, 16
    q = torch.randn(b, n, dk, generator=gen).to(torch.bfloat16)
    keys = (torch.randn(e, m, dk, generator=gen) / 8).to(torch.bfloat16)
    values = torch.randn(e, m, dk, generator=gen).to(torch.bfloat16)
    logits = torch.randn(b, n, e, generator=gen)
    top_l, top_e = logits.topk(2, dim=-1)
    gates = torch.zeros_like(logits).scatter(-1, top_e, torch.softmax(top_l, -1))
    gates[0, 5] = 0.0
    gates[0, 7, 3] = float("nan")
    gates[0, 9, top_e[0, 9, 0]] = 1e-42
    qf, kf, vf, gf = (t.float().numpy() for t in (q, keys, values, gates))
    o, oidx, olse, _ = oracle.gated_mixture_forward(qf, kf, vf, gf, k)
    bias = torch.from_numpy(oracle.gate_bias(gf)).reshape(b * n, e).contiguous()
    out, idx, lse, _ = _ops.topk_attn_fwd(q.reshape(1, b * n, dk).to(DEV), keys.reshape(1, e * m, dk).to(DEV),
                                          values.reshape(1, e * m, dk).to(DEV), k, 1.0, seg_bias=bias.to(DEV))
    assert _native.device_status(clear=True) == 0
    gidx = idx.cpu().numpy().reshape(b * n, k)
    oidx = oidx.reshape(b * n, k)
    special = [5, 7]
    for r in special:
        assert np.array_equal(np.sort(gidx[r]), np.sort(oidx[r])), r
    rest = np.setdiff1d(np.arange(b * n), special)
    sc = np.einsum("nd,md->nm", qf.reshape(-1, dk).astype(np.float64), kf.reshape(-1, dk).astype(np.float64))
    sc = sc + np.repeat(oracle.gate_bias(gf).reshape(b * n, e).astype(np.float64), m, axis=1)
    _assert_indices(gidx[rest][None], oidx[rest][None], sc[rest][None], tol=1e-4, ordered=False,
                    max_near_ties=max(1, len(rest) // 100))
    np.testing.assert_allclose(out.float().cpu().numpy().reshape(b, n, dk), o, rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(lse.cpu().numpy().reshape(b, n), olse, rtol=1e-5, atol=1e-5)


def test_gated_mixture_without_gates_is_flat_top_k():
    from sparsedict_b200 import _ops, gated_mixture_attention

    torch.manual_seed(3)
    q, keys, values = torch.randn(2, 50, 16, device=DEV), torch.randn(3, 40, 16, device=DEV), torch.randn(3, 40, 8, device=DEV)
    out = gated_mixture_attention(q, keys, values, 5)
    flat, _, _, _ = _ops.topk_attn_fwd(q.reshape(1, 100, 16), keys.reshape(1, 120, 16), values.reshape(1, 120, 8), 5, 1.0)
    assert torch.equal(out.reshape(1, 100, 8), flat)


def test_gated_mixture_gradcheck_fp64():
    from sparsedict_b200 import gated_mixture_attention

    torch.manual_seed(9)
    q = torch.randn(1, 6, 5, dtype=torch.float64, device=DEV, requires_grad=True)
    keys = torch.randn(3, 7, 5, dtype=torch.float64, device=DEV, requires_grad=True)
    values = torch.randn(3, 7, 4, dtype=torch.float64, device=DEV, requires_grad=True)
    gates = (torch.rand(1, 6, 3, dtype=torch.float64, device=DEV) + 0.1).requires_grad_(True)
    torch.autograd.gradcheck(lambda *a: gated_mixture_attention(a[0], a[1], a[2], 4, a[3]), (q, keys, values, gates),
                             eps=1e-6, atol=1e-4, nondet_tol=1e-7)


# --- selection operators of models/modules/topk_select.py ------------------------


def test_hard_topk_mask_known_answer(golden):
    from sparsedict_b200 import selection

    masked, idx = selection.hard_topk_mask(_t(golden["known_scores"]), 2)
    assert np.array_equal(idx.cpu().numpy(), golden["known_indices"])
    assert torch.isinf(masked).sum().item() == 4


@pytest.mark.parametrize("mode", ["hard", "ste"])
def test_sparse_topk_attention_configuration_1(golden, mode):
    from sparsedict_b200 import selection

    g = {k[5:]: v for k, v in golden.items() if k.startswith("cfg1_")}
    q, k, v = (_t(g[n]).requires_grad_(True) for n in "qkv")
    scores = (q @ k.transpose(-2, -1)) / math.sqrt(32)
    res = selection.sparse_topk_attention(scores, v, 8, selection=mode)
    np.testing.assert_allclose(res.output.detach().cpu().numpy(), g["out"], atol=1e-5, rtol=0)
    _assert_indices(res.indices.cpu().numpy().reshape(-1, 8), _flat(g["idx"]).reshape(-1, 8),
                    _oracle_scores64(g["q"], g["k"], 1 / math.sqrt(32)).reshape(-1, 128))
    assert res.weights.shape == scores.shape and res.masked_scores.shape == scores.shape
    grads = torch.autograd.grad((res.output * _t(g["do"])).sum(), (q, k, v))
    for got, name in zip(grads, ("dq", "dk", "dv")):
        np.testing.assert_allclose(got.cpu().numpy(), g[name], atol=1e-4, rtol=1e-3)


def test_straight_through_and_gumbel_samples_vs_oracle():
    from sparsedict_b200 import selection

    gen = torch.Generator(device=DEV).manual_seed(5)
    scores = torch.randn(40, 300, device=DEV, generator=gen).requires_grad_(True)
    vals, idx = selection.straight_through_topk(scores, 7)
    ov, oi = oracle.topk_order(scores.detach().cpu().numpy(), 7)
    assert np.array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_array_equal(vals.detach().cpu().numpy(), ov)
    w = torch.randn(40, 7, device=DEV)
    (grad,) = torch.autograd.grad((vals * w).sum(), scores)
    expected = torch.zeros(40, 300, device=DEV).scatter(-1, idx, w)
    assert torch.equal(grad, expected)
    g1 = torch.Generator(device=DEV).manual_seed(123)
    sv, si = selection.gumbel_perturbed_topk(scores.detach(), 7, sigma=0.5, num_samples=3, generator=g1)
    g2 = torch.Generator(device=DEV).manual_seed(123)
    eps = torch.finfo(torch.float32).eps
    for s in range(3):
        u = torch.rand(scores.shape, dtype=torch.float32, device=DEV, generator=g2).clamp(min=eps, max=1 - eps)
        pert = scores.detach() + 0.5 * (-torch.log(-torch.log(u)))
        pv, pi = oracle.topk_order(pert.cpu().numpy(), 7)
        assert np.array_equal(si[s].cpu().numpy(), pi)
        np.testing.assert_array_equal(sv[s].cpu().numpy(), pv)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_straight_through_topk_all_float_dtypes(dtype):
    from sparsedict_b200 import selection

    gen = torch.Generator(device=DEV).manual_seed(8)
    scores = torch.randn(33, 500, device=DEV, generator=gen).to(dtype)
    vals, idx = selection.straight_through_topk(scores, 19)
    assert vals.dtype == dtype
    ov, oi = oracle.topk_order(scores.double().cpu().numpy(), 19)
    assert np.array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_array_equal(vals.double().cpu().numpy(), ov)


# --- deterministic key-major backward ---------------------------------------------


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("bh", "n", "m", "k"), [(2, 384, 1000, 32), (3, 257, 2000, 7), (2, 100, 129, 1),
                                                 (2, 300, 4096, 64), (1, 70, 64, 64)])
def test_key_major_backward_matches_oracle(dtype, bh, n, m, k):
    # The direct backward (dq, dK, dV written once in the input dtype) against
    # the float64 oracle on the support the forward selected.
    from sparsedict_b200 import _ops

    g = torch.Generator().manual_seed(bh * 1000 + n + m + k)
    q, kk, v, do = (torch.randn(bh, x, 64, generator=g).to(dtype).to(DEV) for x in (n, m, m, n))
    scale = 0.125
    _, idx, lse, _ = _ops.topk_attn_fwd(q, kk, v, k, scale)
    dq, dk, dv = _ops.topk_attn_bwd_direct(q, kk, v, do, idx.view(bh, n, k), lse.view(bh, n), scale)
    assert dq.dtype == dk.dtype == dv.dtype == dtype
    assert _native.device_status(clear=True) == 0
    qf, kf, vf, dof = (t.float().cpu().numpy() for t in (q, kk, v, do))
    ref = oracle.topk_attention_backward(qf, kf, vf, idx.view(bh, n, k).cpu().numpy(), dof, scale)
    for got, exp in zip((dq, dk, dv), ref):
        got = got.float().cpu().numpy()
        assert np.abs(got - exp).max() <= 2e-2 * max(1.0, np.abs(exp).max())
    # keys that no row selected get exact zeros
    sel = np.zeros((bh, m), bool)
    np.put_along_axis(sel, idx.view(bh, -1).long().cpu().numpy(), True, axis=1)
    assert not dk.float().cpu().numpy()[~sel].any() and not dv.float().cpu().numpy()[~sel].any()


def test_key_major_backward_is_bitwise_deterministic():
    # dK/dV are written once per key in a fixed summation order: two runs agree
    # bit for bit (the scatter with atomics it replaces does not).
    from sparsedict_b200 import _ops

    g = torch.Generator(device=DEV).manual_seed(99)
    bh, n, m, k = 4, 2048, 4096, 64
    q, kk, v, do = (torch.randn(bh, x, 64, device=DEV, generator=g).to(torch.bfloat16) for x in (n, m, m, n))
    _, idx, lse, _ = _ops.topk_attn_fwd(q, kk, v, k, 0.125)
    idx, lse = idx.view(bh, n, k), lse.view(bh, n)
    first = _ops.topk_attn_bwd_direct(q, kk, v, do, idx, lse, 0.125)
    for _ in range(2):
        again = _ops.topk_attn_bwd_direct(q, kk, v, do, idx, lse, 0.125)
        for a, b in zip(first, again):
            assert torch.equal(a, b)


def test_key_major_backward_skips_given_up_rows():
    # Index -1 (a forward row the bounded wait gave up on) contributes nothing
    # and raises no status bit; the other rows are unaffected.
    from sparsedict_b200 import _ops

    g = torch.Generator(device=DEV).manual_seed(5)
    bh, n, m, k = 2, 256, 1024, 16
    q, kk, v, do = (torch.randn(bh, x, 64, device=DEV, generator=g).to(torch.bfloat16) for x in (n, m, m, n))
    _, idx, lse, _ = _ops.topk_attn_fwd(q, kk, v, k, 0.125)
    idx, lse = idx.view(bh, n, k).clone(), lse.view(bh, n)
    ref = _ops.topk_attn_bwd_direct(q, kk, v, do, idx, lse, 0.125)
    do2 = do.clone()
    do2[0, 7] = 0
    base = _ops.topk_attn_bwd_direct(q, kk, v, do2, idx, lse, 0.125)
    idx[0, 7] = -1
    got = _ops.topk_attn_bwd_direct(q, kk, v, do, idx, lse, 0.125)
    assert _native.device_status(clear=True) == 0
    assert not got[0][0, 7].any()
    assert torch.equal(got[0][:, 8:], ref[0][:, 8:])
    # dK/dV without row 7 = dK/dV with row 7's upstream gradient zeroed (its dS
    # and P·dout are zero there); the per-key lists shift, so not bit for bit
    for a, b in ((got[1], base[1]), (got[2], base[2])):
        assert (a.float() - b.float()).abs().max() <= 1e-2 * max(1.0, float(b.float().abs().max()))


def test_deterministic_switch_routes_autograd_through_key_major_kernels():
    # With the switch on, the public autograd path's dK/dV are bit-identical
    # across runs and equal to the direct key-major entry point's.
    from sparsedict_b200 import _ops, set_deterministic_backward

    g = torch.Generator(device=DEV).manual_seed(41)
    q, kk, v, do = (torch.randn(1, 2, x, 64, device=DEV, generator=g).to(torch.bfloat16) for x in (1024, 2048, 2048, 1024))
    try:
        set_deterministic_backward(True)
        runs = []
        for _ in range(2):
            qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, kk, v))
            out = fused_topk_attention(qd, kd, vd, 32)
            runs.append(torch.autograd.grad(out, (qd, kd, vd), do))
    finally:
        set_deterministic_backward(False)
    for a, b in zip(*runs):
        assert torch.equal(a, b)
    _, idx, lse, _ = _ops.topk_attn_fwd(q.reshape(2, -1, 64), kk.reshape(2, -1, 64), v.reshape(2, -1, 64), 32, 1 / 8)
    ref = _ops.topk_attn_bwd_direct(q.reshape(2, -1, 64), kk.reshape(2, -1, 64), v.reshape(2, -1, 64),
                                    do.reshape(2, -1, 64), idx.view(2, -1, 32), lse.view(2, -1), 1 / 8)
    for a, b in zip(runs[0], ref):
        assert torch.equal(a.reshape(b.shape), b)


def _torch_sparse_attention(scores, values, k):
    # plain torch fp32 restatement of the op, for the gradient check below
    sel, idx = scores.topk(k, dim=-1)
    p = torch.softmax(sel, dim=-1)
    weights = torch.zeros_like(scores).scatter(-1, idx, p)
    masked = torch.full_like(scores, float("-inf")).scatter(-1, idx, sel)
    if values.ndim == 2:
        gathered = values[idx]
    else:
        gathered = torch.stack([values[b][idx[b]] for b in range(values.shape[0])])
    out = (gathered * p.unsqueeze(-1)).sum(-2)
    return out, weights, idx, masked


@pytest.mark.parametrize("batched", [False, True])
def test_sparse_topk_attention_kernels_vs_torch_with_all_gradients(batched):
    # Output, dense weights and masked scores, and the gradients that reach the
    # scores and values through all three, against a plain torch restatement.
    from sparsedict_b200 import selection

    g = torch.Generator(device=DEV).manual_seed(17)
    b, q, m, d, k = 3, 40, 100, 16, 9
    scores = torch.randn(b, q, m, device=DEV, generator=g).requires_grad_(True)
    values = (torch.randn(b, m, d, device=DEV, generator=g) if batched
              else torch.randn(m, d, device=DEV, generator=g)).requires_grad_(True)
    A, B, C = (torch.randn(s, device=DEV, generator=g) for s in ((b, q, d), (b, q, m), (b, q, m)))
    res = selection.sparse_topk_attention(scores, values, k)
    ref = _torch_sparse_attention(scores, values, k)
    assert torch.equal(res.indices, ref[2])
    for got, exp in ((res.output, ref[0]), (res.weights, ref[1]), (res.masked_scores, ref[3])):
        torch.testing.assert_close(got, exp, atol=1e-5, rtol=1e-5)

    def loss(out, weights, masked):
        return (out * A).sum() + (weights * B).sum() + (masked.masked_fill(torch.isinf(masked), 0) * C).sum()

    got = torch.autograd.grad(loss(res.output, res.weights, res.masked_scores), (scores, values))
    exp = torch.autograd.grad(loss(ref[0], ref[1], ref[3]), (scores, values))
    for a, e in zip(got, exp):
        torch.testing.assert_close(a, e, atol=1e-5, rtol=1e-5)


def test_sparse_topk_attention_promotes_mixed_dtypes():
    from sparsedict_b200 import selection

    g = torch.Generator(device=DEV).manual_seed(3)
    scores = torch.randn(50, 64, device=DEV, generator=g).to(torch.bfloat16)
    values = torch.randn(64, 8, device=DEV, generator=g)
    res = selection.sparse_topk_attention(scores, values, 5)
    assert res.output.dtype == torch.float32 and res.weights.dtype == torch.bfloat16
    ref = _torch_sparse_attention(scores.float(), values, 5)
    torch.testing.assert_close(res.output, ref[0], atol=1e-5, rtol=1e-5)
