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

* ``reduce="allreduce"``  all-reduce(SUM) of the full fp32 accumulators
                          (the prescribed exchange, the headline number);
* ``reduce="allgather"``  all-gather of each rank's owned slices;
* ``reduce="none"``       no collective: each rank keeps the gradients of its
                          own slices (sharded).

On CUDA the collective runs in buckets of slices on a side stream, so bucket
``j`` reduces while the backward of bucket ``j+1`` runs.  Every rank issues
the same collectives in the same order.  The compute backend is pluggable
(``kernels``): the default calls the native library; tests substitute a CPU
implementation to exercise the partition and exchange logic on ``gloo``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class ShardPlan:
    """Rows of ``slices`` whole slices split into ``world`` contiguous ranges."""

    slices: int
    world: int
    rank: int

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside a world of {self.world}")
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


class NativeKernels:
    """The CUDA path: fused forward, sparse backward, accumulator conversion."""

    def __init__(self):
        from . import _ops

        self._ops = _ops

    def acc_dtype(self, dtype):
        return self._ops.acc_dtype(dtype)

    def forward(self, q, k, v, topk, scale):
        out, idx, lse, _ = self._ops.topk_attn_fwd(q, k, v, topk, scale)
        return out, idx, lse

    def backward(self, q, k, v, dout, idx, lse, scale, dk_acc, dv_acc, accumulate, dq):
        self._ops.topk_attn_bwd(q, k, v, dout, idx, lse, scale, dk_acc=dk_acc, dv_acc=dv_acc,
                                accumulate=accumulate, dq=dq)

    def finalize(self, acc, dtype):
        return self._ops.finalize_grad(acc, dtype)


class ShardedTopKAttention:
    """Reusable buffers and streams for repeated sharded fwd+bwd steps.

    ``q_rows``/``dout_rows`` hold this rank's slices ``(S/world, N, d)``;
    ``keys``/``values`` are the full replicated ``(S, M, d)`` tensors.
    """

    def __init__(self, plan: ShardPlan, m: int, d: int, dv: int, topk: int, dtype: torch.dtype,
                 device: torch.device, *, temperature: float = 1.0, group=None, reduce: str = "allreduce",
                 buckets: int = 4, kernels=None):
        if reduce not in ("allreduce", "allgather", "none"):
            raise ValueError(f"unknown reduce mode {reduce!r}")
        self.plan, self.m, self.d, self.dv, self.topk = plan, m, d, dv, topk
        self.dtype, self.device, self.group, self.reduce = dtype, torch.device(device), group, reduce
        self.kernels = kernels if kernels is not None else NativeKernels()
        self.scale = 1.0 / (temperature * math.sqrt(d))
        acc = self.kernels.acc_dtype(dtype)
        full = plan.slices if reduce != "none" else plan.per_rank
        self.dk_acc = torch.zeros((full, m, d), device=self.device, dtype=acc)
        self.dv_acc = torch.zeros((full, m, dv), device=self.device, dtype=acc)
        self.buckets = max(1, min(buckets, plan.per_rank)) if plan.world > 1 else 1
        on_cuda = self.device.type == "cuda"
        self.comm_stream = (torch.cuda.Stream(device=self.device)
                            if on_cuda and plan.world > 1 and reduce != "none" else None)

    def _bucket_ranges(self):
        per = self.plan.per_rank
        edges = [round(i * per / self.buckets) for i in range(self.buckets + 1)]
        return [(edges[i], edges[i + 1]) for i in range(self.buckets) if edges[i + 1] > edges[i]]

    def _allreduce_bucket(self, lo, hi):
        # bucket j of every rank, in rank order: the same calls on all ranks
        for r in range(self.plan.world):
            s0 = r * self.plan.per_rank
            dist.all_reduce(self.dk_acc[s0 + lo: s0 + hi], group=self.group)
            dist.all_reduce(self.dv_acc[s0 + lo: s0 + hi], group=self.group)

    def _allgather(self):
        b0, b1 = self.plan.begin, self.plan.end
        own_k = self.dk_acc[b0:b1].clone()
        own_v = self.dv_acc[b0:b1].clone()
        dist.all_gather_into_tensor(self.dk_acc, own_k, group=self.group)
        dist.all_gather_into_tensor(self.dv_acc, own_v, group=self.group)

    def step(self, q_rows, keys, values, dout_rows, fwd_timer=None):
        """Forward and backward of this rank's rows.

        Returns ``(out_rows, dq_rows, dK, dV)``; dK/dV cover all slices
        (replicated) unless ``reduce="none"``, where they cover this rank's.
        ``fwd_timer`` (optional) is a pair of CUDA events recorded around the
        forward kernel.
        """
        plan, kern = self.plan, self.kernels
        b0, b1 = plan.begin, plan.end
        k_loc, v_loc = keys[b0:b1], values[b0:b1]
        if fwd_timer is not None:
            fwd_timer[0].record()
        out, idx, lse = kern.forward(q_rows, k_loc, v_loc, self.topk, self.scale)
        if fwd_timer is not None:
            fwd_timer[1].record()
        exchange = plan.world > 1 and self.reduce != "none"
        local = 0 if self.reduce == "none" else b0
        accumulate = self.reduce == "allreduce" and plan.world > 1
        if accumulate:
            self.dk_acc.zero_()
            self.dv_acc.zero_()
        main = torch.cuda.current_stream(self.device) if self.comm_stream is not None else None
        dq = torch.empty_like(q_rows)
        idx3 = idx.view(plan.per_rank, -1, self.topk)
        lse2 = lse.view(plan.per_rank, -1)
        pending = []
        for lo, hi in self._bucket_ranges():
            kern.backward(q_rows[lo:hi], k_loc[lo:hi], v_loc[lo:hi], dout_rows[lo:hi], idx3[lo:hi], lse2[lo:hi],
                          self.scale, self.dk_acc[local + lo: local + hi], self.dv_acc[local + lo: local + hi],
                          accumulate, dq[lo:hi])
            if exchange and self.reduce == "allreduce":
                if self.comm_stream is not None:
                    ev = torch.cuda.Event()
                    ev.record(main)
                    pending.append((lo, hi, ev))
                else:
                    self._allreduce_bucket(lo, hi)
        if exchange and self.comm_stream is not None:
            with torch.cuda.stream(self.comm_stream):
                if self.reduce == "allreduce":
                    for lo, hi, ev in pending:
                        self.comm_stream.wait_event(ev)
                        self._allreduce_bucket(lo, hi)
                else:
                    self.comm_stream.wait_stream(main)
                    self._allgather()
            main.wait_stream(self.comm_stream)
        elif exchange and self.reduce == "allgather":
            self._allgather()
        dk = kern.finalize(self.dk_acc, self.dtype)
        dv = kern.finalize(self.dv_acc, self.dtype)
        return out, dq, dk, dv
