"""Row-sharded forward + backward over the GPUs of one node.

The partition the workload prescribes: flatten the ``B*H`` slices, give each
rank a contiguous range of whole slices (their query rows), keep keys and
values replicated, and combine the key/value gradients with an NCCL
all-reduce over NVLink in the backward only.  Query rows are independent in
the forward and in dQ, so there is no other exchange.

Because every slice's keys are only ever selected by that slice's own
queries, a rank's dK/dV partials are zero outside its own slices.  The
prescribed all-reduce therefore adds zeros for the other ranks' slices; two
cheaper collectives give the same replicated result or keep it sharded:

* ``reduce="allreduce"``  NCCL all-reduce(SUM) of the full fp32 accumulators
                          (the prescribed exchange, the headline number);
* ``reduce="allgather"``  all-gather of each rank's owned slices;
* ``reduce="none"``       no collective: each rank keeps the gradients of its
                          own slices (sharded).

The collective runs in buckets of slices on a side stream, so bucket ``j``
reduces while the backward of bucket ``j+1`` runs.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _ops


@dataclass
class ShardPlan:
    """Rows of ``slices`` whole slices split into ``world`` contiguous ranges."""

    slices: int
    world: int
    rank: int

    def __post_init__(self):
        if self.slices % self.world:
            raise ValueError(f"{self.slices} slices do not split evenly over {self.world} ranks")

    @property
    def per_rank(self) -> int:
        return self.slices // self.world

    @property
    def begin(self) -> int:
        return self.rank * self.per_rank

    @property
    def end(self) -> int:
        return self.begin + self.per_rank


class ShardedTopKAttention:
    """Reusable buffers and streams for repeated sharded fwd+bwd steps.

    ``q_rows``/``dout_rows`` hold this rank's slices ``(S/world, N, d)``;
    ``keys``/``values`` are the full replicated ``(S, M, d)`` tensors.
    """

    def __init__(self, plan: ShardPlan, m: int, d: int, dv: int, topk: int, dtype: torch.dtype,
                 device: torch.device, *, temperature: float = 1.0, group=None, reduce: str = "allreduce",
                 buckets: int = 4):
        if reduce not in ("allreduce", "allgather", "none"):
            raise ValueError(f"unknown reduce mode {reduce!r}")
        self.plan, self.m, self.d, self.dv, self.topk = plan, m, d, dv, topk
        self.dtype, self.device, self.group, self.reduce = dtype, device, group, reduce
        self.scale = 1.0 / (temperature * math.sqrt(d))
        acc = _ops.acc_dtype(dtype)
        full = plan.slices if reduce != "none" else plan.per_rank
        self.dk_acc = torch.zeros((full, m, d), device=device, dtype=acc)
        self.dv_acc = torch.zeros((full, m, dv), device=device, dtype=acc)
        self.buckets = max(1, min(buckets, plan.per_rank)) if plan.world > 1 else 1
        self.comm_stream = torch.cuda.Stream(device=device) if plan.world > 1 and reduce != "none" else None

    def _bucket_ranges(self):
        per = self.plan.per_rank
        edges = [round(i * per / self.buckets) for i in range(self.buckets + 1)]
        return [(edges[i], edges[i + 1]) for i in range(self.buckets) if edges[i + 1] > edges[i]]

    def step(self, q_rows, keys, values, dout_rows, fwd_timer=None):
        """Forward and backward of this rank's rows.

        Returns ``(out_rows, dq_rows, dK, dV)``; dK/dV cover all slices
        (replicated) unless ``reduce="none"``, where they cover this rank's.
        ``fwd_timer`` (optional) is a pair of CUDA events recorded around the
        forward kernel.
        """
        plan = self.plan
        b0, b1 = plan.begin, plan.end
        k_loc, v_loc = keys[b0:b1], values[b0:b1]
        if fwd_timer is not None:
            fwd_timer[0].record()
        out, idx, lse, _ = _ops.topk_attn_fwd(q_rows, k_loc, v_loc, self.topk, self.scale)
        if fwd_timer is not None:
            fwd_timer[1].record()
        local = 0 if self.reduce == "none" else b0
        if self.reduce == "allreduce" and plan.world > 1:
            self.dk_acc.zero_()
            self.dv_acc.zero_()
        main = torch.cuda.current_stream(self.device)
        dq = torch.empty_like(q_rows)
        work = []
        for lo, hi in self._bucket_ranges():
            _ops.topk_attn_bwd(
                q_rows[lo:hi], k_loc[lo:hi], v_loc[lo:hi], dout_rows[lo:hi], idx.view(plan.per_rank, -1, self.topk)[lo:hi],
                lse.view(plan.per_rank, -1)[lo:hi], self.scale,
                dk_acc=self.dk_acc[local + lo: local + hi], dv_acc=self.dv_acc[local + lo: local + hi],
                accumulate=(self.reduce == "allreduce" and plan.world > 1), dq=dq[lo:hi],
            )
            if self.comm_stream is not None and self.reduce == "allreduce":
                ev = torch.cuda.Event()
                ev.record(main)
                work.append((lo, hi, ev))
        if self.comm_stream is not None:
            with torch.cuda.stream(self.comm_stream):
                if self.reduce == "allreduce":
                    for lo, hi, ev in work:
                        self.comm_stream.wait_event(ev)
                        # the same slice range of every rank: bucket j of all ranks
                        for r in range(plan.world):
                            s0 = r * plan.per_rank
                            dist.all_reduce(self.dk_acc[s0 + lo: s0 + hi], group=self.group)
                            dist.all_reduce(self.dv_acc[s0 + lo: s0 + hi], group=self.group)
                else:  # allgather of owned slices
                    self.comm_stream.wait_stream(main)
                    own_k = self.dk_acc[b0:b1].clone()
                    own_v = self.dv_acc[b0:b1].clone()
                    dist.all_gather_into_tensor(self.dk_acc, own_k, group=self.group)
                    dist.all_gather_into_tensor(self.dv_acc, own_v, group=self.group)
            main.wait_stream(self.comm_stream)
        dk = _ops.finalize_grad(self.dk_acc, self.dtype)
        dv = _ops.finalize_grad(self.dv_acc, self.dtype)
        return out, dq, dk, dv
