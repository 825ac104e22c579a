"""Row-sharded forward + backward over the GPUs of one node.

The partition the workload prescribes: flatten the ``B*H`` slices, give each
rank an equal share of whole slices (their query rows), keep keys and values
replicated, and combine the key/value gradients with an NCCL all-reduce over
NVLink in the backward only.  Query rows are independent in the forward and
in dQ, so there is no other exchange.

Ownership is interleaved by bucket so that the exchanged gradients are
already in slice order.  With ``W`` ranks and ``B`` buckets of ``P`` slices
per rank (``P = S / (W B)``), bucket ``b`` is the contiguous block of slices
``[b W P, (b + 1) W P)`` and rank ``r`` owns its part
``[b W P + r P, b W P + (r + 1) P)``.  (With one bucket this is the plain
contiguous split.)  The step runs bucket by bucket: forward, then the
backward, which writes dK/dV of the rank's slices in the input dtype straight
into its part of the bucket's block of the exchange buffer; the other ranks'
parts of that block are zeroed first.  The block is then all-reduced on a
side stream while the next bucket computes.

Because every slice's keys are only ever selected by that slice's own
queries, a rank's dK/dV are zero outside its own slices: in the all-reduce
every element has exactly one nonzero term, so the sum in the input dtype is
exactly that term (bit-identical to a single process).  Two cheaper
collectives give the same replicated result or keep it sharded:

* ``reduce="allreduce"``  all-reduce(SUM) of each bucket's block (the
                          prescribed exchange, the headline number);
* ``reduce="allgather"``  all-gather of each rank's part of each block;
* ``reduce="none"``       no collective: each rank keeps the gradients of its
                          own slices (sharded, in its local order).

The returned dK/dV are views of the exchange buffer, valid until the next
step.  Every rank issues the same collectives in the same order.  The compute
backend is pluggable (``kernels``): the default calls the native library;
tests substitute a CPU implementation to exercise the partition and exchange
logic on ``gloo``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class ShardPlan:
    """``slices`` whole slices split over ``world`` ranks in ``buckets`` rounds."""

    slices: int
    world: int
    rank: int
    buckets: int = 1

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside a world of {self.world}")
        if self.slices % self.world:
            raise ValueError(f"{self.slices} slices do not split evenly over {self.world} ranks")
        if self.buckets < 1 or self.per_rank % self.buckets:
            raise ValueError(f"{self.per_rank} slices per rank do not split into {self.buckets} buckets")

    @property
    def per_rank(self) -> int:
        return self.slices // self.world

    @property
    def per_bucket(self) -> int:
        """Slices of one rank in one bucket."""
        return self.per_rank // self.buckets

    def block(self, b: int) -> tuple[int, int]:
        """Global slices of bucket ``b`` (all ranks)."""
        w = self.world * self.per_bucket
        return b * w, (b + 1) * w

    def owned_range(self, b: int, rank: int | None = None) -> tuple[int, int]:
        """Global slices of ``rank``'s part of bucket ``b``."""
        r = self.rank if rank is None else rank
        g0 = self.block(b)[0] + r * self.per_bucket
        return g0, g0 + self.per_bucket

    def local_range(self, b: int) -> tuple[int, int]:
        """This rank's local slice indices in bucket ``b``."""
        return b * self.per_bucket, (b + 1) * self.per_bucket

    def global_slice(self, local: int, rank: int | None = None) -> int:
        """Global index of local slice ``local`` of ``rank``."""
        b, i = divmod(local, self.per_bucket)
        return self.owned_range(b, rank)[0] + i

    def owned(self, rank: int | None = None) -> list[int]:
        return [self.global_slice(i, rank) for i in range(self.per_rank)]


def pick_buckets(slices: int, world: int, want: int) -> int:
    """The largest bucket count <= ``want`` that divides the per-rank slices."""
    per = max(1, slices // world)
    for b in range(max(1, min(want, per)), 0, -1):
        if per % b == 0:
            return b
    return 1


class NativeKernels:
    """The CUDA path: fused forward and the direct (input-dtype) backward."""

    def __init__(self):
        from . import _ops

        self._ops = _ops

    def forward(self, q, k, v, topk, scale, out):
        out, idx, lse, _ = self._ops.topk_attn_fwd(q, k, v, topk, scale, out=out)
        return out, idx, lse

    def backward(self, q, k, v, dout, idx, lse, scale, dq, dk, dv):
        self._ops.topk_attn_bwd_out(q, k, v, dout, idx, lse, scale, dq=dq, dk=dk, dv=dv)


class ShardedTopKAttention:
    """Reusable buffers and streams for repeated sharded fwd+bwd steps.

    ``q_rows``/``dout_rows`` hold this rank's slices in local order
    ``(S/world, N, d)`` (local slice ``i`` is global slice
    ``plan.global_slice(i)``); ``keys``/``values`` are the full replicated
    ``(S, M, d)`` tensors.
    """

    def __init__(self, plan: ShardPlan, m: int, d: int, dv: int, topk: int, dtype: torch.dtype,
                 device: torch.device, *, temperature: float = 1.0, group=None, reduce: str = "allreduce",
                 kernels=None):
        if reduce not in ("allreduce", "allgather", "none"):
            raise ValueError(f"unknown reduce mode {reduce!r}")
        self.plan, self.m, self.d, self.dv, self.topk = plan, m, d, dv, topk
        self.dtype, self.device, self.group, self.reduce = dtype, torch.device(device), group, reduce
        self.kernels = kernels if kernels is not None else NativeKernels()
        self.scale = 1.0 / (temperature * math.sqrt(d))
        exchange = plan.world > 1 and reduce != "none"
        full = plan.slices if reduce != "none" else plan.per_rank
        # the exchange buffer (reduce != "none", slice order) or the rank's own gradients
        self.grad_k = torch.zeros((full, m, d), device=self.device, dtype=dtype)
        self.grad_v = torch.zeros((full, m, dv), device=self.device, dtype=dtype)
        on_cuda = self.device.type == "cuda"
        # high priority: the exchange kernels take SMs as the backward's blocks retire
        self.comm_stream = (torch.cuda.Stream(device=self.device, priority=-1)
                            if on_cuda and exchange else None)

    @property
    def launches_per_step(self) -> int:
        """Kernels of this library per step: per bucket the forward (stream +
        finishing kernel) and the backward (the scatter kernel and two
        conversions, or with the deterministic backward the row, transpose and
        key kernels)."""
        return self.plan.buckets * 5

    def _dst(self, b):
        if self.reduce == "none":
            lo, hi = self.plan.local_range(b)
            return self.grad_k[lo:hi], self.grad_v[lo:hi]
        g0, g1 = self.plan.owned_range(b)
        return self.grad_k[g0:g1], self.grad_v[g0:g1]

    def _clear_others(self, b):
        # the other ranks' parts of the block must be zero for the sum
        b0, b1 = self.plan.block(b)
        g0, g1 = self.plan.owned_range(b)
        for t in (self.grad_k, self.grad_v):
            if g0 > b0:
                t[b0:g0].zero_()
            if b1 > g1:
                t[g1:b1].zero_()

    def _exchange(self, b):
        b0, b1 = self.plan.block(b)
        if self.reduce == "allreduce":
            dist.all_reduce(self.grad_k[b0:b1], group=self.group)
            dist.all_reduce(self.grad_v[b0:b1], group=self.group)
        else:
            g0, g1 = self.plan.owned_range(b)
            for t in (self.grad_k, self.grad_v):
                dist.all_gather_into_tensor(t[b0:b1], t[g0:g1].clone(), group=self.group)

    def step(self, q_rows, keys, values, dout_rows, fwd_timer=None):
        """Forward and backward of this rank's rows, bucket by bucket.

        Returns ``(out_rows, dq_rows, dK, dV)``; dK/dV cover all slices in
        slice order (replicated) unless ``reduce="none"``, where they cover
        this rank's slices in local order.  ``fwd_timer`` (optional) is a list
        to which a pair of CUDA events around each bucket's forward is
        appended.
        """
        plan, kern = self.plan, self.kernels
        exchange = plan.world > 1 and self.reduce != "none"
        on_cuda = self.device.type == "cuda"
        main = torch.cuda.current_stream(self.device) if self.comm_stream is not None else None
        out = torch.empty((*q_rows.shape[:-1], self.dv), device=q_rows.device, dtype=q_rows.dtype)
        dq = torch.empty_like(q_rows)
        for b in range(plan.buckets):
            lo, hi = plan.local_range(b)
            g0, g1 = plan.owned_range(b)
            k_b, v_b = keys[g0:g1], values[g0:g1]
            if fwd_timer is not None and on_cuda:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            _, idx, lse = kern.forward(q_rows[lo:hi], k_b, v_b, self.topk, self.scale, out[lo:hi])
            if fwd_timer is not None and on_cuda:
                ev[1].record()
                fwd_timer.append(ev)
            if exchange and self.reduce == "allreduce":
                self._clear_others(b)
            dk, dv = self._dst(b)
            kern.backward(q_rows[lo:hi], k_b, v_b, dout_rows[lo:hi], idx.view(hi - lo, -1, self.topk),
                          lse.view(hi - lo, -1), self.scale, dq[lo:hi], dk, dv)
            if exchange:
                if self.comm_stream is not None:
                    done = torch.cuda.Event()
                    done.record(main)
                    with torch.cuda.stream(self.comm_stream):
                        self.comm_stream.wait_event(done)
                        self._exchange(b)
                else:
                    self._exchange(b)
        if exchange and self.comm_stream is not None:
            main.wait_stream(self.comm_stream)
        return out, dq, self.grad_k, self.grad_v
