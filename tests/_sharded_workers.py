"""Worker processes for the gloo (CPU) tests of the sharded step.

The compute backend here is built from the CPU oracle, so these processes
exercise only the partition and exchange logic of ``sparsedict_b200.sharded``.
"""

import os
import traceback
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

import oracle
from sparsedict_b200.sharded import ShardedTopKAttention, ShardPlan

S, N, M, D, TOPK = 8, 24, 40, 8, 5


class OracleKernels:
    def forward(self, q, k, v, topk, scale, out):
        o, idx, lse, _ = oracle.topk_attention_forward(q.numpy(), k.numpy(), v.numpy(), topk, scale)
        out.copy_(torch.from_numpy(o))
        return out, torch.from_numpy(idx).reshape(-1, topk), torch.from_numpy(lse).reshape(-1)

    def backward(self, q, k, v, dout, idx, lse, scale, dq, dk, dv):
        gq, gk, gv = oracle.topk_attention_backward(q.numpy(), k.numpy(), v.numpy(), idx.numpy(), dout.numpy(), scale)
        dq.copy_(torch.from_numpy(gq))
        dk.copy_(torch.from_numpy(gk))
        dv.copy_(torch.from_numpy(gv))


def inputs():
    rng = np.random.default_rng(7)
    q, k, v, do = (torch.from_numpy(rng.standard_normal(shape)) for shape in
                   ((S, N, D), (S, M, D), (S, M, D), (S, N, D)))
    return q, k, v, do


def run_rank(rank, world, port, reduce, fail_rank, results):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        q, k, v, do = inputs()
        plan = ShardPlan(S, world, rank, buckets=2)
        runner = ShardedTopKAttention(plan, M, D, D, TOPK, torch.float64, "cpu", reduce=reduce,
                                      kernels=OracleKernels())
        if rank == fail_rank:
            raise RuntimeError("injected failure before the backward exchange")
        own = plan.owned()
        out, dq, dk, dv = runner.step(q[own].contiguous(), k, v, do[own].contiguous())
        results.put(("ok", rank, out.numpy(), dq.numpy(), dk.numpy(), dv.numpy()))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, which asserts on it
        results.put(("error", rank, f"{type(exc).__name__}: {exc}", traceback.format_exc()))
