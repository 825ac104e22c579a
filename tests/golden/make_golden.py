"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in the development container, where the reference checkout is
importable (it does not exist on GPU machines, which only read the
committed ``.npz`` files):

    python tests/golden/make_golden.py --reference /root/reference

Every expected output below comes from the reference's own PyTorch code:
``models.modules.topk_select.sparse_topk_attention`` (with torch autograd
for gradients) and ``torch.topk``.  Inputs are drawn with torch's CPU
generator so they are reproducible from the recorded seeds; they are stored
in the fixtures as well, except for the one large parity grid whose inputs
are regenerated from its seed and checked against a stored checksum.
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def _reference_scores(q, k, temperature=1.0):
    # tests/test_triton_autograd.py:40-46 and tests/test_hybrid_topk.py:245-248
    return (q @ k.transpose(-2, -1)) / (temperature * math.sqrt(q.shape[-1]))


def _fwd_bwd(sparse_topk_attention, q, k, v, dout, topk):
    q = q.detach().clone().requires_grad_(True)
    k = k.detach().clone().requires_grad_(True)
    v = v.detach().clone().requires_grad_(True)
    res = sparse_topk_attention(_reference_scores(q, k), v, topk)
    grads = torch.autograd.grad((res.output * dout).sum(), (q, k, v))
    return res, grads


def big_case_inputs(seed, n, m, dk, dv):
    torch.manual_seed(seed)
    q = torch.randn(1, 1, n, dk)
    k = torch.randn(1, 1, m, dk)
    v = torch.randn(1, 1, m, dv)
    return q, k, v


def checksum(*arrays) -> float:
    return float(sum(np.float64(np.abs(a).sum()) for a in arrays))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from models.modules.topk_select import hard_topk_mask, sparse_topk_attention

    out: dict[str, np.ndarray] = {}
    out["meta_torch_version"] = np.array(torch.__version__)

    # known answer, tests/test_topk_select.py:13-19
    scores = torch.tensor([[1.0, 4.0, 2.0, 3.0], [8.0, 5.0, 7.0, 6.0]])
    _, idx = hard_topk_mask(scores, k=2)
    out["known_scores"] = _np(scores)
    out["known_indices"] = _np(idx)

    # configuration 1: B=1, H=2, N=256, M=128, d=32, k=8, seed 0, fp32 fwd+bwd
    torch.manual_seed(0)
    q = torch.randn(1, 2, 256, 32)
    k = torch.randn(1, 2, 128, 32)
    v = torch.randn(1, 2, 128, 32)
    do = torch.randn(1, 2, 256, 32)
    res, (gq, gk, gv) = _fwd_bwd(sparse_topk_attention, q, k, v, do, 8)
    for name, t in dict(q=q, k=k, v=v, do=do, out=res.output, idx=res.indices,
                        dq=gq, dk=gk, dv=gv).items():
        out[f"cfg1_{name}"] = _np(t)

    # forward parity grids, tests/test_triton_autograd.py:63-75 (d=64, seed 1234)
    grids = [(1, 13, 1, 24), (7, 64, 5, 67), (65, 129, 17, 33), (3, 73, 73, 7)]
    for n, m, kk, dv in grids:
        q, k, v = big_case_inputs(1234, n, m, 64, dv)
        res = sparse_topk_attention(_reference_scores(q, k), v, kk)
        tag = f"grid_{n}_{m}_{kk}_{dv}"
        out[f"{tag}_q"], out[f"{tag}_k"], out[f"{tag}_v"] = _np(q), _np(k), _np(v)
        out[f"{tag}_out"] = _np(res.output)
        out[f"{tag}_idx"] = _np(res.indices)
    # the large grid: inputs regenerated from the seed, outputs stored strided
    n, m, kk, dv = 4096, 256, 16, 64
    q, k, v = big_case_inputs(1234, n, m, 64, dv)
    res = sparse_topk_attention(_reference_scores(q, k), v, kk)
    tag = "grid_4096_256_16_64"
    out[f"{tag}_checksum"] = np.array(checksum(_np(q), _np(k), _np(v)))
    out[f"{tag}_out_rows8"] = _np(res.output)[..., ::8, :]
    out[f"{tag}_idx"] = _np(res.indices).astype(np.int16)

    # float64 forward, tests/test_triton_autograd.py:78-86
    torch.manual_seed(1234)
    q = torch.randn(1, 2, 32, 8, dtype=torch.float64)
    k = torch.randn(1, 2, 24, 8, dtype=torch.float64)
    v = torch.randn(1, 2, 24, 6, dtype=torch.float64)
    res = sparse_topk_attention(_reference_scores(q, k), v, 5)
    for name, t in dict(q=q, k=k, v=v, out=res.output, idx=res.indices).items():
        out[f"f64fwd_{name}"] = _np(t)

    # float64 backward vs autograd, tests/test_triton_autograd.py:141-173
    torch.manual_seed(42)
    q = torch.randn(2, 3, 32, 8, dtype=torch.float64)
    k = torch.randn(2, 3, 24, 8, dtype=torch.float64)
    v = torch.randn(2, 3, 24, 6, dtype=torch.float64)
    w = torch.randn(2, 3, 32, 6, dtype=torch.float64)
    res, (gq, gk, gv) = _fwd_bwd(sparse_topk_attention, q, k, v, w, 7)
    for name, t in dict(q=q, k=k, v=v, do=w, out=res.output, idx=res.indices,
                        dq=gq, dk=gk, dv=gv).items():
        out[f"f64bwd_{name}"] = _np(t)

    # hybrid forward grids, tests/test_hybrid_topk.py:251-266 (seed 101)
    for b, h, n, m, dk, dv, kk in [(1, 1, 7, 129, 8, 5, 7), (2, 2, 5, 263, 16, 33, 11)]:
        torch.manual_seed(101)
        q = torch.randn(b, h, n, dk)
        k = torch.randn(b, h, m, dk)
        v = torch.randn(b, h, m, dv)
        res = sparse_topk_attention(_reference_scores(q, k), v, kk)
        tag = f"hyb_{b}_{h}_{n}_{m}_{dk}_{dv}_{kk}"
        out[f"{tag}_q"], out[f"{tag}_k"], out[f"{tag}_v"] = _np(q), _np(k), _np(v)
        out[f"{tag}_out"] = _np(res.output)
        out[f"{tag}_idx"] = _np(res.indices)

    # hybrid autograd, tests/test_hybrid_topk.py:269-293 (seed 202)
    torch.manual_seed(202)
    q = torch.randn(1, 2, 9, 8)
    k = torch.randn(1, 2, 137, 8)
    v = torch.randn(1, 2, 137, 6)
    do = torch.randn(1, 2, 9, 6)
    res, (gq, gk, gv) = _fwd_bwd(sparse_topk_attention, q, k, v, do, 5)
    for name, t in dict(q=q, k=k, v=v, do=do, out=res.output, idx=res.indices,
                        dq=gq, dk=gk, dv=gv).items():
        out[f"hybgrad_{name}"] = _np(t)

    # tiled_topk exact indices, tests/test_fused_topk_attn.py:106-139
    for rows, keys, kk in [(1, 1, 1), (7, 64, 5), (65, 129, 17), (8, 256, 64), (3, 73, 73)]:
        gen = torch.Generator().manual_seed(rows * 10000 + keys * 100 + kk)
        rnd = torch.rand((rows, keys), generator=gen)
        sc = rnd.argsort(dim=1).argsort(dim=1).to(torch.float32)
        vals, idx = torch.topk(sc, kk, dim=1)
        tag = f"topk_{rows}_{keys}_{kk}"
        out[f"{tag}_scores"], out[f"{tag}_vals"], out[f"{tag}_idx"] = _np(sc), _np(vals), _np(idx)

    # tiled_topk_aggregate, tests/test_fused_topk_attn.py:142-189
    for qc, kc, kk, dv in [(1, 13, 1, 24), (7, 64, 5, 67), (65, 129, 17, 33), (3, 73, 73, 7)]:
        gen = torch.Generator().manual_seed(qc * 10000 + kc * 100 + kk + dv)
        sc = torch.randn((qc, kc), generator=gen)
        vals = torch.randn((kc, dv), generator=gen)
        ts, ti = torch.topk(sc, kk, dim=1)
        weights = torch.softmax(ts.float(), dim=1)
        expected = torch.sum(weights.unsqueeze(-1) * vals.float()[ti], dim=1)
        tag = f"agg_{qc}_{kc}_{kk}_{dv}"
        out[f"{tag}_scores"], out[f"{tag}_values"] = _np(sc), _np(vals)
        out[f"{tag}_ts"], out[f"{tag}_ti"], out[f"{tag}_out"] = _np(ts), _np(ti), _np(expected)

    # routed dictionary attention (configuration 3 at a small size): the gate
    # fold of models/modules/dual_domain_moe.py:158-173 with top-1 gates from
    # models/modules/router.py:139-145, then the reference sparse_topk_attention.
    torch.manual_seed(3)
    n, d, e, m, kk = 512, 16, 4, 64, 8
    qm = torch.randn(1, n, d)
    atoms = torch.randn(e, m, d) / math.sqrt(d)
    logits = torch.randn(1, n, e)
    dom = torch.randn(1, n, d)
    sel_logits, sel_exp = logits.topk(1, dim=-1)
    gates = torch.zeros_like(logits).scatter(-1, sel_exp, torch.softmax(sel_logits, -1))
    qg = qm.clone().requires_grad_(True)
    ag = atoms.clone().requires_grad_(True)
    scores = torch.einsum("bnk,emk->bnem", qg, ag)
    tiny = torch.finfo(scores.dtype).tiny
    scores = scores + gates.clamp_min(tiny).log().unsqueeze(-1)
    scores = scores.masked_fill(gates.unsqueeze(-1) == 0, float("-inf"))
    scores = scores.reshape(1, n, e * m)
    res = sparse_topk_attention(scores, ag.reshape(e * m, d), kk)
    gq, ga = torch.autograd.grad((res.output * dom).sum(), (qg, ag))
    for name, t in dict(q=qm[0], atoms=atoms, logits=logits[0], do=dom[0],
                        out=res.output[0], flat_idx=res.indices[0],
                        dq=gq[0], datoms=ga).items():
        out[f"moe_{name}"] = _np(t)

    # gated mixture (models/modules/dual_domain_moe.py:139-174) with soft gates:
    # separate key and value projections of the atoms, gates from top-2 softmax
    # routing for half of the tokens (zeros elsewhere) and dense softmax gates
    # for the rest, gradients into queries, keys, values and gates.
    torch.manual_seed(5)
    b, n, dk, c, e, m, kk = 2, 48, 16, 12, 4, 40, 9
    qm = torch.randn(b, n, dk)
    keys = torch.randn(e, m, dk) / math.sqrt(dk)
    values = torch.randn(e, m, c)
    logits = torch.randn(b, n, e)
    top_l, top_e = logits.topk(2, dim=-1)
    sparse_g = torch.zeros_like(logits).scatter(-1, top_e, torch.softmax(top_l, -1))
    dense_g = torch.softmax(logits, -1)
    gates = torch.where((torch.arange(n) % 2 == 0).view(1, n, 1), sparse_g, dense_g)
    dom = torch.randn(b, n, c)
    qg, kg, vg, gg = (t.clone().requires_grad_(True) for t in (qm, keys, values, gates))
    scores = torch.einsum("bnk,emk->bnem", qg, kg)
    tiny = torch.finfo(scores.dtype).tiny
    scores = scores + gg.clamp_min(tiny).log().unsqueeze(-1)
    scores = scores.masked_fill(gg.unsqueeze(-1) == 0, float("-inf"))
    scores = scores.reshape(b, n, e * m)
    res = sparse_topk_attention(scores, vg.reshape(e * m, c), kk)
    gq, gkeys, gvalues, ggates = torch.autograd.grad((res.output * dom).sum(), (qg, kg, vg, gg))
    for name, t in dict(q=qm, keys=keys, values=values, gates=gates, do=dom, out=res.output,
                        flat_idx=res.indices, dq=gq, dkeys=gkeys, dvalues=gvalues, dgates=ggates).items():
        out[f"mix_{name}"] = _np(t)

    path = HERE / "reference_vectors.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size / 1024:.0f} KiB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
