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
from sparsedict_b200.sharded import ShardedTopKAttention, ShardPlan, pick_buckets


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
    # one bucket: the plain contiguous split
    plans = [ShardPlan(128, 8, r) for r in range(8)]
    assert [p.owned() for p in plans] == [list(range(16 * r, 16 * r + 16)) for r in range(8)]
    # four buckets: bucket b is slices [32b, 32b + 32), rank r owns [32b + 4r, 32b + 4r + 4)
    plans = [ShardPlan(128, 8, r, buckets=4) for r in range(8)]
    assert plans[3].owned() == [32 * b + 12 + i for b in range(4) for i in range(4)]
    assert plans[3].block(2) == (64, 96) and plans[3].owned_range(2) == (76, 80)
    assert plans[3].local_range(2) == (8, 12) and plans[3].global_slice(9) == 77
    with pytest.raises(ValueError):
        ShardPlan(10, 4, 0)
    with pytest.raises(ValueError):
        ShardPlan(8, 2, 2)
    with pytest.raises(ValueError):
        ShardPlan(16, 2, 0, buckets=3)
    assert pick_buckets(128, 8, 4) == 4 and pick_buckets(24, 4, 4) == 3 and pick_buckets(8, 8, 4) == 1


@pytest.mark.parametrize("reduce", ["allreduce", "allgather", "none"])
def test_two_ranks_match_single_process(reduce):
    res, _ = _run(2, reduce)
    assert all(r[0] == "ok" for r in res), [r[2:] for r in res if r[0] != "ok"]
    q, k, v, do = (t.numpy() for t in W.inputs())
    scale = 1 / np.sqrt(W.D)
    o, idx, _, _ = oracle.topk_attention_forward(q, k, v, W.TOPK, scale)
    gq, gk, gv = oracle.topk_attention_backward(q, k, v, idx, do, scale)
    for _, rank, out, dq, dk, dv in res:
        rows = ShardPlan(W.S, 2, rank, buckets=2).owned()
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


@pytest.mark.parametrize("slices,world,buckets", [(16, 2, 4), (48, 8, 2), (18, 3, 2), (128, 8, 4), (7, 7, 1)])
def test_bucket_interleaved_ownership_is_a_partition(slices, world, buckets):
    # every global slice is owned by exactly one (rank, local slice); bucket b
    # of all ranks is one contiguous block in slice order and each rank's part
    # of it is contiguous, so the exchanged buffer needs no reordering
    seen = {}
    for rank in range(world):
        plan = ShardPlan(slices, world, rank, buckets=buckets)
        for b in range(buckets):
            b0, b1 = plan.block(b)
            g0, g1 = plan.owned_range(b)
            lo, hi = plan.local_range(b)
            assert b0 <= g0 < g1 <= b1 and g1 - g0 == hi - lo
            for i in range(lo, hi):
                g = plan.global_slice(i)
                assert g == g0 + i - lo and g not in seen
                seen[g] = (rank, i)
    assert sorted(seen) == list(range(slices))
