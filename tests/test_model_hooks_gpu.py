"""The model hooks against the dense attention path of SparseDict's models.

The stand-in module has the attributes the reference's ``_mixture``
(models/modules/dual_domain_moe.py:139-174) reads — ``projections[branch]``
with ``query``/``key``/``value`` layers and ``_atom_projections`` — and a
dense ``_mixture`` restated in torch (scores for every atom, the gate fold,
top-k, softmax over the selected scores, value sum).  Binding the fused hook
must give the same outputs and gradients.
"""

import math

import numpy as np
import pytest
import torch

from sparsedict_b200 import fused_token_attention, install_fused_mixture

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _dense_topk_attention(scores, values, k):
    top, idx = scores.topk(k, dim=-1)
    w = torch.softmax(top, dim=-1)
    return torch.einsum("bnk,bnkc->bnc", w, values[idx])


def _fold(scores, gates):
    tiny = torch.finfo(scores.dtype).tiny
    scores = scores + gates.clamp_min(tiny).log().unsqueeze(-1)
    return scores.masked_fill(gates.unsqueeze(-1) == 0, float("-inf"))


class _Dictionary(torch.nn.Module):
    def __init__(self, c, dk):
        super().__init__()
        self.projections = torch.nn.ModuleList([torch.nn.ModuleDict({
            "query": torch.nn.Linear(c, dk),
            "key": torch.nn.Linear(c, dk, bias=False),
            "value": torch.nn.Linear(c, c, bias=False),
        })])

    def _atom_projections(self, branch, bank):
        proj = self.projections[branch]
        keys = torch.einsum("emc,kc->emk", bank, proj["key"].weight)
        values = torch.einsum("emc,fc->emf", bank, proj["value"].weight)
        return keys, values

    def _mixture(self, query_tokens, branch, bank, top_k, gates=None):
        q = self.projections[branch]["query"](query_tokens)
        keys, values = self._atom_projections(branch, bank)
        scores = torch.einsum("bnk,emk->bnem", q, keys)
        if gates is not None:
            scores = _fold(scores, gates)
        b, n, e, m = scores.shape
        return _dense_topk_attention(scores.reshape(b, n, e * m), values.reshape(e * m, -1), top_k)


@pytest.mark.parametrize("with_gates", [False, True])
def test_fused_mixture_hook_matches_dense_mixture(with_gates):
    torch.manual_seed(3)
    b, n, c, dk, e, m, k = 2, 96, 32, 16, 4, 40, 8
    mod = _Dictionary(c, dk).to(DEV)
    tokens = torch.randn(b, n, c, device=DEV, requires_grad=True)
    bank = torch.randn(e, m, c, device=DEV, requires_grad=True)
    gates = None
    if with_gates:
        logits = torch.randn(b, n, e, device=DEV)
        top_l, top_e = logits.topk(2, dim=-1)
        gates = torch.zeros_like(logits).scatter(-1, top_e, torch.softmax(top_l, -1))
    dout = torch.randn(b, n, c, device=DEV)
    ref = mod._mixture(tokens, 0, bank, k, gates)
    g_ref = torch.autograd.grad((ref * dout).sum(), (tokens, bank))
    install_fused_mixture(mod)
    out = mod._mixture(tokens, 0, bank, k, gates)
    g_out = torch.autograd.grad((out * dout).sum(), (tokens, bank))
    np.testing.assert_allclose(out.detach().cpu().numpy(), ref.detach().cpu().numpy(), atol=1e-4, rtol=1e-4)
    for got, exp in zip(g_out, g_ref):
        np.testing.assert_allclose(got.cpu().numpy(), exp.cpu().numpy(), atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("dtype,dk,m,tol", [(torch.float32, 16, 40, 1e-4), (torch.bfloat16, 64, 128, 2e-2)])
def test_fused_token_attention_matches_scaled_dense_fold(dtype, dk, m, tol):
    # (q·k + log g) / (tau * sqrt(d_k)) with -inf where g == 0, top-k over the
    # flat atoms; bf16 with d_k = 64 and 128-atom experts takes the
    # tensor-core forward with the gate bias
    g = torch.Generator().manual_seed(7)
    b, n, e, k, tau = 2, 200, 4, 16, 0.7
    q = torch.randn(b, n, dk, generator=g)
    keys = torch.randn(e, m, dk, generator=g) / 4
    values = torch.randn(e, m, 32 if dtype == torch.float32 else 64, generator=g)
    logits = torch.randn(b, n, e, generator=g)
    top_l, top_e = logits.topk(2, dim=-1)
    gates = torch.zeros_like(logits).scatter(-1, top_e, torch.softmax(top_l, -1))
    qd, kd, vd, gd = (t.to(DEV, dtype).requires_grad_(True) for t in (q, keys, values, gates))
    out = fused_token_attention(qd, kd, vd, gd, k, tau)
    dout = torch.randn(out.shape, generator=g).to(DEV, dtype)
    grads = torch.autograd.grad((out.float() * dout.float()).sum(), (qd, kd, vd, gd))
    qr, kr, vr, gr = (t.detach().double().requires_grad_(True) for t in (qd, kd, vd, gd))
    scores = _fold(torch.einsum("bnk,emk->bnem", qr, kr), gr) / (tau * math.sqrt(dk))
    ref = _dense_topk_attention(scores.reshape(b, n, e * m), vr.reshape(e * m, -1), k)
    refg = torch.autograd.grad((ref * dout.double()).sum(), (qr, kr, vr, gr))
    np.testing.assert_allclose(out.detach().double().cpu().numpy(), ref.detach().cpu().numpy(), atol=tol, rtol=tol)
    for got, exp in zip(grads, refg):
        got, exp = got.double().cpu().numpy(), exp.cpu().numpy()
        assert np.abs(got - exp).max() <= tol * max(1.0, np.abs(exp).max())
