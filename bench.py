#!/usr/bin/env python
"""Throughput of fused top-k sparse attention, forward + backward, on B200.

Workload (the headline configuration): B=16, H=8, N=M=16384 tokens, d=64,
k=64, bf16 inputs with fp32 accumulation; Q, K, V, dO iid N(0,1) from a
seed.  A step is one forward and one backward over all B*H*N query rows,
split as whole (b, h) slices across the ranks with K and V replicated and the
fp32 dK/dV accumulators all-reduced over NVLink (strong scaling: the total
work is fixed).  Inputs (268 MB each) are larger than the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU
restatement of the reference path (dense scores, hard top-k, softmax,
gather, dense autograd-style backward) on this host's cores instead.

``--workload routed`` measures the dictionary-MoE configuration instead:
N=16384 tokens, d=64, 8 experts of M=1024 atoms (keys = values), top-1
routing by the argmax of N(0,1) router logits, k=16 within the expert, bf16
forward and backward through ``routed_dictionary_attention`` (one replica
per GPU: the routed op is not sharded).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "top-k attn fwd+bwd queries/sec @1/2/4/8 B200; % tensor-pipe & HBM roofline"
UNIT = "queries/s"
CFG = dict(B=16, H=8, N=16384, M=16384, d=64, k=64)
WORKLOAD = "sharded bf16 fwd+bwd, B=16 H=8 N=M=16384 d=64 k=64"
ROUTED_METRIC = "routed top-k dictionary attn fwd+bwd queries/sec (B200)"
ROUTED_CFG = dict(N=16384, d=64, E=8, M=1024, k=16)
ROUTED_WORKLOAD = "routed dictionary bf16 fwd+bwd, N=16384 tokens d=64, E=8 experts x M=1024 atoms, top-1, k=16"
L2_FLUSH_BYTES = 256 << 20


def roofline_terms(b, h, n, m, d, k, elem):
    """Algorithmic work of one fwd+bwd over all slices: the dense affinity flops and
    the compulsory HBM bytes (read Q, K, V, dO; write O, dQ, dK, dV; indices and LSE)."""
    flops_tc = 2.0 * n * m * d * b * h  # the dense affinity, the only dense contraction
    bytes_fb = ((5 * n + 6 * m) * d * elem + 8 * n * (k + 1)) * b * h
    return flops_tc, bytes_fb


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic():
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            return {}
    return {}


class ClockSampler:
    """SM clock and throttle-reason samples taken while the timed region runs.

    Polls NVML (read-only queries) every 2 ms from a thread, so that even a
    timed region of a few milliseconds gets samples; falls back to
    ``nvidia-smi --query-gpu`` every 25 ms when NVML is not importable.
    Entering waits for the first sample and drops it, so every kept sample
    was taken inside the region.
    """

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event-reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, index, device=None):
        self.index = index
        self.device = device
        self.proc = None
        self.lines = []
        self.samples = []  # (sm_mhz, max_mhz, reason_bits)
        self._stop = threading.Event()
        self._nvml = None

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        handle = None
        try:
            import torch

            bus = torch.cuda.get_device_properties(self.device).pci_bus_id
            dom = torch.cuda.get_device_properties(self.device).pci_domain_id
            dev = torch.cuda.get_device_properties(self.device).pci_device_id
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev:02x}.0".encode())
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        mx = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        return pynvml, handle, reasons, mx

    def _poll(self):
        nv, handle, reasons, mx = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM), mx, reasons(handle)))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        try:
            self._nvml = self._nvml_handle()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            deadline = time.monotonic() + 5.0
            while not self.samples and time.monotonic() < deadline:
                time.sleep(0.001)
            self.samples.clear()
            return self
        except Exception:
            self._nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "25"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            deadline = time.monotonic() + 5.0
            while not self.lines and time.monotonic() < deadline and self.proc.poll() is None:
                time.sleep(0.005)
            self.lines.clear()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self.thread.join(timeout=1)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        for clk, cmax, bits in self.samples:
            sm.append(float(clk))
            mx = float(cmax)
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        src = "nvml" if self._nvml is not None else "nvidia-smi"
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0, "source": src}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": src}


# ----------------------------------------------------------------- CPU arms --


def cpu_reference_sample(rows=256, seed=0):
    """Time the CPU restatement of the reference path on one bounded slice.

    One (b, h) slice of the workload: ``rows`` query rows against all M keys
    (bf16-rounded inputs, fp32 compute), forward and backward.  Returns
    (queries/s, seconds, description).
    """
    import numpy as np

    import oracle

    c = CFG
    rng = np.random.default_rng(seed)
    q = oracle.round_to_bf16(rng.standard_normal((1, rows, c["d"]), dtype=np.float32))
    k = oracle.round_to_bf16(rng.standard_normal((1, c["M"], c["d"]), dtype=np.float32))
    v = oracle.round_to_bf16(rng.standard_normal((1, c["M"], c["d"]), dtype=np.float32))
    do = rng.standard_normal((1, rows, c["d"]), dtype=np.float32)
    t0 = time.perf_counter()
    oracle.dense_reference_fwd_bwd(q, k, v, do, c["k"], 1 / math.sqrt(c["d"]))
    dt = time.perf_counter() - t0
    return rows / dt, dt, f"one (b,h) slice: {rows} query rows x M={c['M']} keys, d={c['d']}, k={c['k']}, fp32 " \
                          "on bf16-rounded inputs, dense fwd+bwd; queries/s extrapolated from the slice"


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_reference_sample(rows=args.ref_rows)
    rates, secs = [], []
    for i in range(args.steps):
        r, s, desc = cpu_reference_sample(rows=args.ref_rows, seed=i + 1)
        rates.append(r)
        secs.append(s)
    value = statistics.median(rates)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * statistics.median(secs),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, **CFG, "sample_rows": args.ref_rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- GPU arm --


def run_e2e(args, c, world, dev, runner, tensors, barrier, total_queries):
    """Same metric end to end through the public API, host buffers on both sides.

    Every step copies its inputs (this rank's query and upstream-gradient
    rows, the replicated keys and values) from pinned host memory, runs the
    forward and backward, and copies every result (output and dQ rows, dK,
    dV) back into pinned host memory.  Input copies of step i+1 run on a copy
    stream while step i computes; result copies of step i run on a third
    stream while step i+1 computes.  At one GPU the API is
    ``fused_topk_attention`` + autograd, at several the sharded step
    (``ShardedTopKAttention.step``).
    """
    import torch
    import torch.distributed as dist

    from sparsedict_b200 import fused_topk_attention

    host = [t.cpu().pin_memory() for t in tensors]
    h2d = sum(t.numel() * t.element_size() for t in host)
    main = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(device=dev)
    back_stream = torch.cuda.Stream(device=dev)
    bufs = [[torch.empty_like(t, device=dev) for t in host] for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    q_rows, keys, values, dout_rows = tensors
    # pinned result buffers: out and dQ of this rank's rows, dK and dV
    res_host = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q_rows, q_rows, keys, values)]
    d2h = sum(t.numel() * t.element_size() for t in res_host)

    def issue_copy(slot):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[slot])
            for dst, src in zip(bufs[slot], host):
                dst.copy_(src, non_blocking=True)
            copied[slot].record(copy_stream)

    def compute(slot):
        main.wait_event(copied[slot])
        qd, kd, vd, dod = bufs[slot]
        if world == 1:
            qd4, kd4, vd4 = (x.view(c["B"], c["H"], -1, c["d"]).requires_grad_(True) for x in (qd, kd, vd))
            out = fused_topk_attention(qd4, kd4, vd4, c["k"])
            dq, dk, dv = torch.autograd.grad(out, (qd4, kd4, vd4), dod.view_as(out))
        else:
            out, dq, dk, dv = runner.step(qd, kd, vd, dod)
        consumed[slot].record(main)
        results = (out, dq, dk, dv)
        back_stream.wait_stream(main)
        with torch.cuda.stream(back_stream):
            for dst, src in zip(res_host, results):
                dst.copy_(src.reshape(dst.shape), non_blocking=True)
        for t in results:
            t.record_stream(back_stream)

    def run(steps):
        for ev in consumed:
            ev.record(main)
        issue_copy(0)
        for i in range(steps):
            if i + 1 < steps:
                issue_copy((i + 1) % 2)
            compute(i % 2)
        back_stream.synchronize()

    run(max(1, args.warmup))
    barrier()
    t0 = time.perf_counter()
    run(args.e2e_steps)
    barrier()
    e2e_s = torch.tensor([time.perf_counter() - t0], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    return {"value": total_queries * args.e2e_steps / float(e2e_s[0]), "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": args.e2e_steps,
            "note": "public API; every step copies its inputs from pinned host memory and copies out, dQ, dK "
                    "and dV back into pinned host memory (input copies overlap the previous step's compute, "
                    "result copies the next step's); bytes are per rank"}


def check_parity(c, world, rank, dev, plan, runner, keys, values, q_rows, dout_rows, rows=256):
    """Sharded results against a one-process recomputation, outside the timed region.

    Each rank recomputes one of its own slices, and (at several GPUs) one
    slice of the next rank — whose query and gradient rows it regenerates
    from that rank's seed — with the single-GPU public API
    (``fused_topk_attention`` + autograd on that slice alone), and compares
    sampled rows of the sharded step's output and dQ (own slice) and of the
    all-reduced dK and dV (both slices).  The forward must match bit for bit;
    gradients within the bf16 tolerance.  All ranks take part in the same
    reductions, so the verdict is global.
    """
    import torch
    import torch.distributed as dist

    from sparsedict_b200 import fused_topk_attention

    out, dq, dk, dv = runner.step(q_rows, keys, values, dout_rows)
    torch.cuda.synchronize(dev)
    gen = torch.Generator(device=dev)
    sel = torch.Generator().manual_seed(7)
    worst = {"out": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
    exact_out = True
    checked = []
    owners = [rank] + ([(rank + 1) % world] if world > 1 else [])
    for owner in owners:
        local = 0 if owner == rank else plan.per_rank - 1
        s = plan.global_slice(local, owner)
        if owner == rank:
            qs, dos = q_rows[local], dout_rows[local]
        else:
            gen.manual_seed(1234 + 1000 * (owner + 1))
            qa = torch.randn(plan.per_rank, c["N"], c["d"], device=dev, generator=gen).to(q_rows.dtype)
            da = torch.randn(plan.per_rank, c["N"], c["d"], device=dev, generator=gen).to(q_rows.dtype)
            qs, dos = qa[local], da[local]
        q4, k4, v4 = (t.reshape(1, 1, -1, c["d"]).clone().requires_grad_(True) for t in (qs, keys[s], values[s]))
        ref_out = fused_topk_attention(q4, k4, v4, c["k"])
        rdq, rdk, rdv = torch.autograd.grad(ref_out, (q4, k4, v4), dos.reshape(ref_out.shape))
        r_idx = torch.randperm(c["N"], generator=sel)[:rows].to(dev)
        k_idx = torch.randperm(c["M"], generator=sel)[:rows].to(dev)

        def err(a, b):
            a, b = a.float(), b.float()
            return float((a - b).abs().max()) / max(1.0, float(b.abs().max()))

        if owner == rank:
            got_out = out[local][r_idx]
            exact_out &= bool(torch.equal(got_out, ref_out.reshape(-1, c["d"])[r_idx]))
            worst["out"] = max(worst["out"], err(got_out, ref_out.reshape(-1, c["d"])[r_idx]))
            worst["dq"] = max(worst["dq"], err(dq[local][r_idx], rdq.reshape(-1, c["d"])[r_idx]))
        dks, dvs = (dk[s], dv[s]) if runner.reduce != "none" else (dk[local], dv[local])
        if runner.reduce != "none" or owner == rank:
            worst["dk"] = max(worst["dk"], err(dks[k_idx], rdk.reshape(-1, c["d"])[k_idx]))
            worst["dv"] = max(worst["dv"], err(dvs[k_idx], rdv.reshape(-1, c["d"])[k_idx]))
        checked.append(s)
    t = torch.tensor([worst["out"], worst["dq"], worst["dk"], worst["dv"], 0.0 if exact_out else 1.0],
                     device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    worst = dict(zip(("out", "dq", "dk", "dv"), (float(x) for x in t[:4])))
    ok = float(t[4]) == 0.0 and all(v <= 2e-2 for v in worst.values())
    return {"ok": ok, "forward_bit_exact": float(t[4]) == 0.0, "max_rel_err": worst, "tolerance": 2e-2,
            "checked": f"{rows} sampled rows of out/dQ (own slice) and of dK/dV (own slice"
                       + (" and one slice of the next rank" if world > 1 else "") + ") against the single-GPU "
                       "public API on that slice alone"}


def routed_inputs(torch, dev, seed=1234):
    c = ROUTED_CFG
    gen = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(c["N"], c["d"], generator=gen).to(torch.bfloat16)
    atoms = (torch.randn(c["E"], c["M"], c["d"], generator=gen) / math.sqrt(c["d"])).to(torch.bfloat16)
    logits = torch.randn(c["N"], c["E"], generator=gen)
    do = torch.randn(c["N"], c["d"], generator=gen).to(torch.bfloat16)
    return q, atoms, logits, do


def cpu_routed_sample(tokens=ROUTED_CFG["N"], seed=0):
    """The CPU restatement of the routed path on ``tokens`` tokens of the workload
    (all 8 dictionaries), forward and backward.  Returns (queries/s, seconds, description)."""
    import numpy as np

    import oracle

    c = ROUTED_CFG
    rng = np.random.default_rng(seed)
    q = oracle.round_to_bf16(rng.standard_normal((tokens, c["d"]), dtype=np.float32))
    atoms = oracle.round_to_bf16(rng.standard_normal((c["E"], c["M"], c["d"]), dtype=np.float32) / 8)
    logits = rng.standard_normal((tokens, c["E"]), dtype=np.float32)
    do = rng.standard_normal((tokens, c["d"]), dtype=np.float32)
    t0 = time.perf_counter()
    experts = oracle.moe_route_top1(logits)
    _, idx, _ = oracle.moe_topk_attention_forward(q, atoms, experts, c["k"], 1.0)
    oracle.moe_topk_attention_backward(q, atoms, experts, idx, do, 1.0)
    dt = time.perf_counter() - t0
    return tokens / dt, dt, f"{tokens} tokens routed over E={c['E']} dictionaries of M={c['M']} atoms, d={c['d']}, " \
                            f"k={c['k']}, fp32 on bf16-rounded inputs, fwd+bwd" + \
        ("" if tokens == c["N"] else "; queries/s extrapolated")


def tensor_peak_key(clock_summary):
    """The burst bf16 peak is the denominator for a step that keeps the maximum SM
    clock (the forward runs for milliseconds inside a sub-second loop); a clock
    record that shows the power cap, or a median clock well below the maximum,
    selects the sustained figure measured under the cap."""
    capped = "sw_power_cap" in (clock_summary.get("reasons") or []) or (
        clock_summary.get("sm_mhz") and clock_summary.get("sm_max_mhz")
        and clock_summary["sm_mhz"] < 0.9 * clock_summary["sm_max_mhz"])
    return "bf16_tflops_sustained" if capped else "bf16_tflops"


def run_routed_arm(args):
    import torch
    import torch.distributed as dist

    from sparsedict_b200 import _native, routed_dictionary_attention

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        for _ in range(args.warmup):
            cpu_routed_sample()
        rates, secs = [], []
        for i in range(args.steps):
            r, sec, desc = cpu_routed_sample(seed=i + 1)
            rates.append(r)
            secs.append(sec)
        value = statistics.median(rates)
        print(json.dumps({
            "metric": ROUTED_METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * statistics.median(secs),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": ROUTED_WORKLOAD, **ROUTED_CFG},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
                             "sample": desc},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _native.load()
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    c = ROUTED_CFG
    hq, ha, hl, hd = routed_inputs(torch, dev)
    q = hq.to(dev).requires_grad_(True)
    atoms = ha.to(dev).requires_grad_(True)
    logits, do = hl.to(dev), hd.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step():
        out = routed_dictionary_attention(q, atoms, logits, c["k"], 1.0)
        return (out,) + torch.autograd.grad(out, (q, atoms), grad_outputs=do)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(local, dev) as clocks:
        barrier()
        for i in range(args.steps):
            flush.fill_(i & 0xFF)  # evict the previous step's inputs and outputs from L2 (outside the events)
            ev[i][0].record(stream)
            out = routed_dictionary_attention(q, atoms, logits, c["k"], 1.0)
            ev[i][1].record(stream)
            torch.autograd.grad(out, (q, atoms), grad_outputs=do)
            ev[i][2].record(stream)
        barrier()
    elapsed = sum(e[0].elapsed_time(e[2]) for e in ev) / 1000.0
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    t = torch.tensor([elapsed, fwd_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed, fwd_ms = float(t[0]), float(t[1])
    value = world * c["N"] * args.steps / elapsed

    e2e = None
    if not args.skip_e2e:
        # public API end to end: pinned host inputs in, fwd+bwd, O, dQ and dDict back to pinned host
        pins = [t.pin_memory() for t in (hq, ha, hl, hd)]
        outs = [torch.empty((c["N"], c["d"]), dtype=torch.bfloat16).pin_memory(),
                torch.empty((c["N"], c["d"]), dtype=torch.bfloat16).pin_memory(),
                torch.empty((c["E"], c["M"], c["d"]), dtype=torch.bfloat16).pin_memory()]
        h2d = sum(t.numel() * t.element_size() for t in pins)
        d2h = sum(t.numel() * t.element_size() for t in outs)

        def e2e_step():
            dq_, da_, dl, dd = (t.to(dev, non_blocking=True) for t in pins)
            dq_.requires_grad_(True)
            da_.requires_grad_(True)
            o = routed_dictionary_attention(dq_, da_, dl, c["k"], 1.0)
            g = torch.autograd.grad(o, (dq_, da_), grad_outputs=dd)
            for h, dsrc in zip(outs, (o.detach(), g[0], g[1])):
                h.copy_(dsrc, non_blocking=True)

        for _ in range(3):
            e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        et = torch.tensor([e0.elapsed_time(e1) / 1000.0], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": world * c["N"] * args.e2e_steps / float(et[0]), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "sparsedict_b200.routed_dictionary_attention + torch.autograd.grad"}

    peaks = load_peaks()
    flops = 2.0 * c["N"] * c["M"] * c["d"]  # each token against the M atoms of its expert
    achieved = flops / (fwd_ms / 1000.0) / 1e12
    clock_summary = clocks.summary()
    peak_key = tensor_peak_key(clock_summary)
    peak_tc = peaks[peak_key]
    line = {
        "metric": ROUTED_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": ROUTED_WORKLOAD, **c, "parallelism": f"replicas{world}",
                   "l2": f"flushed between steps ({L2_FLUSH_BYTES >> 20} MB write outside the timed events)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tc, "unit": "TFLOP/s",
                     "frac": achieved / peak_tc, "traffic": None,
                     "kernel": "forward (routing + stream + finish kernels)", "fwd_ms": fwd_ms,
                     "peak_source": f"{peaks['source']} {peak_key}"},
        # per step: the router's count, scan and place kernels, the forward's stream
        # and finishing kernels, the backward's scatter kernel and the
        # dictionary-gradient conversion
        "gpu_launches": 7 * args.steps,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if rank == 0 and not args.skip_cpu:
        r, sec, desc = cpu_routed_sample()
        line["cpu_baseline"] = {"value": r, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": desc}
    line["clocks"] = clock_summary
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def run_native_arm(args):
    import torch
    import torch.distributed as dist

    from sparsedict_b200 import _native
    from sparsedict_b200.sharded import ShardedTopKAttention, ShardPlan, pick_buckets

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _native.load()
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        group = dist.group.WORLD

    c = dict(CFG, B=args.batch, H=args.heads)
    slices = c["B"] * c["H"]
    plan = ShardPlan(slices, world, rank, buckets=pick_buckets(slices, world, args.buckets) if world > 1 else 1)
    gen = torch.Generator(device=dev).manual_seed(1234)
    dtype = torch.bfloat16
    keys = torch.randn(slices, c["M"], c["d"], device=dev, generator=gen).to(dtype)
    values = torch.randn(slices, c["M"], c["d"], device=dev, generator=gen).to(dtype)
    gen.manual_seed(1234 + 1000 * (rank + 1))
    q_rows = torch.randn(plan.per_rank, c["N"], c["d"], device=dev, generator=gen).to(dtype)
    dout_rows = torch.randn(plan.per_rank, c["N"], c["d"], device=dev, generator=gen).to(dtype)
    runner = ShardedTopKAttention(plan, c["M"], c["d"], c["d"], c["k"], dtype, dev, group=group,
                                  reduce=args.reduce)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        runner.step(q_rows, keys, values, dout_rows)
    barrier()

    stream = torch.cuda.current_stream(dev)
    fwd_events = [[] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, dev) as clocks:
        barrier()
        start.record(stream)
        for i in range(args.steps):
            runner.step(q_rows, keys, values, dout_rows, fwd_timer=fwd_events[i])
        stop.record(stream)
        barrier()
    elapsed = start.elapsed_time(stop) / 1000.0
    # forward time per step: the sum over the step's buckets
    fwd_ms = statistics.mean(sum(a.elapsed_time(b) for a, b in evs) for evs in fwd_events)
    t = torch.tensor([elapsed, fwd_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed, fwd_ms = float(t[0]), float(t[1])

    total_queries = slices * c["N"]
    value = total_queries * args.steps / elapsed
    ms_per_step = 1000 * elapsed / args.steps

    # end to end through the public API: pinned host inputs copied in, fwd+bwd,
    # a scalar result read back, every step (the rank's own rows).  The input
    # copies of step i+1 run on a second stream into the other of two device
    # buffer sets while step i computes, as a training loader would.
    e2e = None
    if not args.skip_e2e:
        e2e = run_e2e(args, c, world, dev, runner, (q_rows, keys, values, dout_rows), barrier, total_queries)

    parity = None
    if not args.skip_parity:
        parity = check_parity(c, world, rank, dev, plan, runner, keys, values, q_rows, dout_rows)

    peaks = load_peaks()
    flops_tc, bytes_fb = roofline_terms(c["B"], c["H"], c["N"], c["M"], c["d"], c["k"], 2)
    # dominant kernels: the forward (streaming kernel: affinity MMA + selection;
    # finishing kernel: exact re-score, softmax, value gather), one call = two launches
    fwd_flops_per_launch = flops_tc / world
    achieved = fwd_flops_per_launch / (fwd_ms / 1000.0) / 1e12
    clock_summary = clocks.summary()
    peak_key = tensor_peak_key(clock_summary)
    peak_tc = peaks[peak_key]
    # ncu-measured DRAM bytes of one headline forward call (profiles/traffic.json)
    traffic = load_traffic().get("forward_B16_H8_N16384_k64") if (c["B"], c["H"], world) == (CFG["B"], CFG["H"], 1) else None
    t_tensor = flops_tc / world / (peak_tc * 1e12)
    t_hbm = bytes_fb / world / (peaks["hbm_gbs"] * 1e9)
    t_roof = max(t_tensor, t_hbm)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD if (args.batch, args.heads) == (CFG["B"], CFG["H"]) else
                   f"sharded bf16 fwd+bwd, B={args.batch} H={args.heads} N=M=16384 d=64 k=64",
                   **c, "parallelism": f"rows{world}", "reduce": args.reduce,
                   "l2": "inputs larger than L2 (268 MB per tensor)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tc, "unit": "TFLOP/s",
                     "frac": achieved / peak_tc, "traffic": traffic, "kernel": "forward (stream + finish kernels)",
                     "fwd_ms": fwd_ms, "peak_source": f"{peaks['source']} {peak_key}",
                     "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
                     "step_frac_combined": t_roof / (ms_per_step / 1000.0),
                     # each whole-step term on its own: affinity flops at the tensor peak,
                     # compulsory fwd+bwd bytes at the HBM peak
                     "step_frac_tensor": t_tensor / (ms_per_step / 1000.0),
                     "step_frac_hbm": t_hbm / (ms_per_step / 1000.0)},
        # this library's kernels per step: per bucket the forward (stream + finishing
        # kernel) and the backward kernels
        "gpu_launches": runner.launches_per_step * args.steps,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if parity is not None:
        line["parity"] = parity
    if rank == 0 and not args.skip_cpu:
        r, s, desc = cpu_reference_sample(rows=args.ref_rows)
        rates = [r]
        budget = time.perf_counter() + 10
        i = 1
        while time.perf_counter() < budget and i < 8:
            rates.append(cpu_reference_sample(rows=args.ref_rows, seed=i)[0])
            i += 1
        line["cpu_baseline"] = {"value": statistics.median(rates), "unit": UNIT, "cores": os.cpu_count() or 1,
                                "kind": "port", "sample": desc + f"; median of {len(rates)}"}
    line["clocks"] = clock_summary
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--reduce", choices=["allreduce", "allgather", "none"], default="allreduce")
    ap.add_argument("--buckets", type=int, default=4)
    ap.add_argument("--batch", type=int, default=CFG["B"], help="B (default: the headline 16)")
    ap.add_argument("--heads", type=int, default=CFG["H"], help="H (default: the headline 8)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--ref-rows", type=int, default=256)
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-parity", action="store_true")
    ap.add_argument("--workload", choices=["sharded", "routed"], default="sharded")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "routed":
        return run_routed_arm(args)
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_native_arm(args)


if __name__ == "__main__":
    sys.exit(main())
