"""Per-query adaptive k against a dense float64 restatement.

Row (b, h, n) attends over its own k_i best keys (larger score first, lower
index on ties); the expected result masks every other score of a dense
q·kᵀ·scale row to -inf before the softmax, in float64 with torch autograd.
"""

import math

import numpy as np
import pytest
import torch

from sparsedict_b200 import _native, _ops, adaptive_topk_attention, fused_topk_attention

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _dense_reference(q, k, v, kq, scale, do):
    q, k, v = (t.detach().double().cpu().requires_grad_(True) for t in (q, k, v))
    s = torch.einsum("bhnd,bhmd->bhnm", q, k) * scale
    # reference order: larger score first, lower key index on ties (stable sort)
    order = torch.sort(-s.detach(), dim=-1, stable=True).indices
    rank = torch.empty_like(order)
    rank.scatter_(-1, order, torch.arange(s.shape[-1]).expand_as(order))
    keep = rank < kq.cpu().long().unsqueeze(-1)
    p = torch.softmax(s.masked_fill(~keep, float("-inf")), dim=-1)
    out = torch.einsum("bhnm,bhmd->bhnd", p, v)
    grads = torch.autograd.grad((out * do.double().cpu()).sum(), (q, k, v))
    return out.detach(), grads, keep


@pytest.mark.parametrize("dtype,d,m,k_max,tol", [(torch.float32, 32, 300, 16, 1e-4),
                                                  (torch.bfloat16, 64, 1000, 32, 2e-2)])
def test_adaptive_topk_matches_dense_masked_softmax(dtype, d, m, k_max, tol):
    g = torch.Generator().manual_seed(d + m + k_max)
    b, h, n = 2, 2, 200
    q, kk, v, do = (torch.randn(b, h, x, d, generator=g) for x in (n, m, m, n))
    kq = torch.randint(1, k_max + 1, (b, h, n), generator=g, dtype=torch.int32)
    kq[0, 0, :3] = torch.tensor([1, k_max, k_max])
    qd, kd, vd = (t.to(DEV, dtype).requires_grad_(True) for t in (q, kk, v))
    out = adaptive_topk_attention(qd, kd, vd, kq.to(DEV), k_max=k_max)
    grads = torch.autograd.grad((out.float() * do.to(DEV)).sum(), (qd, kd, vd))
    assert _native.device_status(clear=True) == 0
    scale = 1 / math.sqrt(d)
    ref, ref_grads, keep = _dense_reference(qd, kd, vd, kq, scale, do)
    np.testing.assert_allclose(out.detach().double().cpu().numpy(), ref.numpy(), atol=tol, rtol=tol)
    for got, exp in zip(grads, ref_grads):
        got, exp = got.double().cpu().numpy(), exp.numpy()
        assert np.abs(got - exp).max() <= tol * max(1.0, np.abs(exp).max())
    # the selected index sets: row r lists its k_i keys, then -1
    _, idx, _, _ = _ops.topk_attn_fwd(qd.detach().reshape(b * h, n, d), kd.detach().reshape(b * h, m, d),
                                      vd.detach().reshape(b * h, m, d), k_max, scale,
                                      row_k=kq.reshape(-1).to(DEV))
    idx = idx.cpu().numpy().reshape(b, h, n, k_max)
    want = keep.numpy()
    agree = 0
    for bb in range(b):
        for hh in range(h):
            for r in range(n):
                kr = int(kq[bb, hh, r])
                assert (idx[bb, hh, r, kr:] == -1).all()
                got_set = set(idx[bb, hh, r, :kr].tolist())
                agree += got_set == set(np.nonzero(want[bb, hh, r])[0].tolist())
    # fp32 selects exactly; bf16 may swap keys within rounding of the k-th score
    assert agree >= (b * h * n if dtype == torch.float32 else int(0.98 * b * h * n))


@pytest.mark.parametrize("dtype,d", [(torch.float32, 32), (torch.bfloat16, 64)])
def test_adaptive_topk_with_full_budget_is_the_fused_op(dtype, d):
    torch.manual_seed(4)
    q, kk, v = (torch.randn(1, 2, x, d, device=DEV).to(dtype) for x in (130, 700, 700))
    kq = torch.full((1, 2, 130), 24, dtype=torch.int32, device=DEV)
    assert torch.equal(adaptive_topk_attention(q, kk, v, kq), fused_topk_attention(q, kk, v, 24))
