"""Host logic of the row-sharded step on two gloo ranks (CPU).

The partition (whole slices per rank), the bucketed all-reduce, the
all-gather of owned slices and the no-exchange mode must all reproduce a
single-process computation; a rank that fails before the exchange must make
its peer's collective fail within the process-group timeout instead of
hanging.
"""

import multiprocessing as mp
import socket
import time

import numpy as np
import pytest
import torch

import _sharded_workers as W
import oracle
from sparsedict_b200.sharded import ShardedTopKAttention, ShardPlan


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, reduce, fail_rank=-1, limit=60):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=W.run_rank, args=(r, world, port, reduce, fail_rank, results)) for r in range(world)]
    t0 = time.time()
    for p in procs:
        p.start()
    out = []
    for _ in procs:
        out.append(results.get(timeout=limit))
    for p in procs:
        p.join(timeout=limit)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not exit")
    return sorted(out, key=lambda r: r[1]), time.time() - t0


def test_shard_plan_splits_whole_slices():
    plans = [ShardPlan(128, 8, r) for r in range(8)]
    assert [(p.begin, p.end) for p in plans] == [(16 * r, 16 * r + 16) for r in range(8)]
    with pytest.raises(ValueError):
        ShardPlan(10, 4, 0)
    with pytest.raises(ValueError):
        ShardPlan(8, 2, 2)


@pytest.mark.parametrize("reduce", ["allreduce", "allgather", "none"])
def test_two_ranks_match_single_process(reduce):
    res, _ = _run(2, reduce)
    assert all(r[0] == "ok" for r in res), [r[2:] for r in res if r[0] != "ok"]
    q, k, v, do = (t.numpy() for t in W.inputs())
    scale = 1 / np.sqrt(W.D)
    o, idx, _, _ = oracle.topk_attention_forward(q, k, v, W.TOPK, scale)
    gq, gk, gv = oracle.topk_attention_backward(q, k, v, idx, do, scale)
    per = W.S // 2
    for _, rank, out, dq, dk, dv in res:
        rows = slice(rank * per, (rank + 1) * per)
        np.testing.assert_allclose(out, o[rows], atol=1e-12)
        np.testing.assert_allclose(dq, gq[rows], atol=1e-12)
        if reduce == "none":
            np.testing.assert_allclose(dk, gk[rows], atol=1e-12)
            np.testing.assert_allclose(dv, gv[rows], atol=1e-12)
        else:
            np.testing.assert_allclose(dk, gk, atol=1e-12)
            np.testing.assert_allclose(dv, gv, atol=1e-12)


def test_failed_rank_makes_peer_collective_fail_not_hang():
    res, elapsed = _run(2, "allreduce", fail_rank=1, limit=60)
    assert res[1][0] == "error" and "injected" in res[1][2]
    assert res[0][0] == "error", "the surviving rank should see its collective fail"
    assert elapsed < 55


@pytest.mark.parametrize("slices,world,buckets", [(16, 2, 4), (40, 8, 2), (15, 3, 2), (128, 8, 4), (7, 7, 3)])
def test_bucket_major_layout_is_a_bijection(slices, world, buckets):
    # every (rank, local slice) maps to its own accumulator row, bucket j of all
    # ranks is one contiguous block, and each rank's part of it is contiguous
    class _Kernels:
        def acc_dtype(self, dtype):
            return torch.float32

    seen = {}
    for rank in range(world):
        runner = ShardedTopKAttention(ShardPlan(slices, world, rank), 4, 2, 2, 1, torch.float32, "cpu",
                                      reduce="allreduce", buckets=buckets, kernels=_Kernels())
        assert runner._bucket_major == (world > 1)
        for lo, hi in runner._bucket_ranges():
            a0, a1 = runner._acc_range(lo, hi, rank)
            assert a1 - a0 == hi - lo
            if world > 1:
                assert world * lo <= a0 and a1 <= world * hi
            for i, row in enumerate(range(a0, a1)):
                assert row not in seen
                seen[row] = (rank, lo + i)
    assert sorted(seen) == list(range(slices))
