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
``j`` reduces while the backward of bucket ``j+1`` runs.  For the all-reduce
the fp32 accumulators are laid out bucket-major, ``[bucket][rank][slice]``:
a rank's slices of one bucket stay contiguous for the kernel, and bucket
``j`` of every rank forms one contiguous block that a single all-reduce call
covers (two calls per bucket, not two per rank per bucket).  Each rank
converts its own part of a bucket to the output dtype in a staging block whose
other ranks' parts are zero, and the staging block is what is all-reduced:
every element has exactly one nonzero term, so the sum in the output dtype is
bit-identical to converting the fp32 sum, at half the bytes for bf16.  A last
copy puts dK/dV back in slice order.  Every rank issues the same
collectives in the same order.  The compute backend is pluggable
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

    def finalize(self, acc, dtype, out=None):
        return self._ops.finalize_grad(acc, dtype, out=out)


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
        if self._bucket_major:
            self.stage_k = torch.zeros((full, m, d), device=self.device, dtype=dtype)
            self.stage_v = torch.zeros((full, m, dv), device=self.device, dtype=dtype)
        on_cuda = self.device.type == "cuda"
        # high priority: the exchange kernels take SMs as the backward's blocks retire
        self.comm_stream = (torch.cuda.Stream(device=self.device, priority=-1)
                            if on_cuda and plan.world > 1 and reduce != "none" else None)

    def _bucket_ranges(self):
        per = self.plan.per_rank
        edges = [round(i * per / self.buckets) for i in range(self.buckets + 1)]
        return [(edges[i], edges[i + 1]) for i in range(self.buckets) if edges[i + 1] > edges[i]]

    @property
    def _bucket_major(self) -> bool:
        return self.reduce == "allreduce" and self.plan.world > 1

    def _acc_range(self, lo, hi, rank):
        """Accumulator rows of ``rank``'s local slices ``[lo, hi)``."""
        if self._bucket_major:
            # bucket [lo, hi) of all ranks starts at world*lo; rank r's part follows r blocks of hi-lo
            a0 = self.plan.world * lo + rank * (hi - lo)
            return a0, a0 + (hi - lo)
        local = 0 if self.reduce == "none" else rank * self.plan.per_rank
        return local + lo, local + hi

    def _allreduce_bucket(self, lo, hi):
        # bucket j of every rank is one contiguous block: the same calls on all ranks
        w = self.plan.world
        dist.all_reduce(self.stage_k[w * lo: w * hi], group=self.group)
        dist.all_reduce(self.stage_v[w * lo: w * hi], group=self.group)

    def _slice_order(self, stage):
        out = torch.empty_like(stage)
        per = self.plan.per_rank
        for lo, hi in self._bucket_ranges():
            for r in range(self.plan.world):
                a0, a1 = self._acc_range(lo, hi, r)
                out[r * per + lo: r * per + hi].copy_(stage[a0:a1])
        return out

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
        if self._bucket_major:
            # the other ranks' parts of each staging block must be zero for the sum
            self.stage_k.zero_()
            self.stage_v.zero_()
        main = torch.cuda.current_stream(self.device) if self.comm_stream is not None else None
        dq = torch.empty_like(q_rows)
        idx3 = idx.view(plan.per_rank, -1, self.topk)
        lse2 = lse.view(plan.per_rank, -1)
        pending = []
        for lo, hi in self._bucket_ranges():
            a0, a1 = self._acc_range(lo, hi, plan.rank)
            kern.backward(q_rows[lo:hi], k_loc[lo:hi], v_loc[lo:hi], dout_rows[lo:hi], idx3[lo:hi], lse2[lo:hi],
                          self.scale, self.dk_acc[a0:a1], self.dv_acc[a0:a1], False, dq[lo:hi])
            if self._bucket_major:
                kern.finalize(self.dk_acc[a0:a1], self.dtype, out=self.stage_k[a0:a1])
                kern.finalize(self.dv_acc[a0:a1], self.dtype, out=self.stage_v[a0:a1])
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
        if self._bucket_major:
            return out, dq, self._slice_order(self.stage_k), self._slice_order(self.stage_v)
        dk = kern.finalize(self.dk_acc, self.dtype)
        dv = kern.finalize(self.dv_acc, self.dtype)
        return out, dq, dk, dv
