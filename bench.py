#!/usr/bin/env python
"""Benchmark of the B200 batched token sampler.

Default workload: the mixed-parameter continuous batch (B=64, V=151936,
bf16 logits, per-row temperature / top_k / top_p / min_p / presence /
frequency / repetition penalties over a 1024-token Zipf history), sampled
with in-kernel Philox draws and in-kernel history / RNG-offset updates, i.e.
one decode step of the sampler as it runs inside a captured decode graph.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

ours:       K steps replayed from CUDA graphs over rotating logits buffers whose
            total size exceeds 2x the 126 MB L2 (every step reads cold HBM);
            CUDA-event timing on the launching stream, max over ranks.
            roofline: algorithmic bytes / the kernel's mean launch duration over
            the timed region (events around every single launch, captured in a
            second graph, are reported beside it); e2e: the same steps through
            the public Python API from pinned host logits (H2D + step + D2H of
            the ids inside the timed region).
reference:  the CPU restatement of the sampler spec (oracle/, C + OpenMP) on
            the host cores, rank 0 only, on a bounded sample of the workload.
Multi-GPU (torchrun): data-parallel replicas, each rank samples its own batch
(weak scaling, no collective on the data path).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled rows/sec + ncu HBM GB/s (% of peak) at B=64, V=151936 bf16"
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="qwen_mixed",
                    choices=["qwen_mixed", "orpheus_single", "bucket", "constrained", "tp"])
    ap.add_argument("--bucket", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cluster", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=200)
    return ap.parse_args()


def make_case(args, rank):
    from mstar_rs_b200 import workloads as W

    if args.workload == "qwen_mixed":
        return W.qwen_mixed(seed=args.seed + rank)
    if args.workload == "orpheus_single":
        return W.orpheus_single(seed=args.seed + rank)
    if args.workload == "bucket":
        return W.bucket_sweep(args.bucket, seed=args.seed + rank)
    if args.workload == "tp":  # the reference arm samples the whole row (vocab sharding is ours)
        return W.tp_full(W.tp_sharded(1, seed=args.seed))
    return W.constrained(seed=args.seed + rank)


def algorithmic_bytes(case) -> int:
    """One read of the logits, the penalty / bias / mask inputs and the
    per-slot parameters, plus the writes of ids and per-slot state."""
    es = 2 if case.dtype == "bf16" else 4
    b = case.B * case.V * es
    if case.hist_ids is not None:
        b += case.hist_ids.nbytes + case.hist_len.nbytes
        b += case.B * 8  # history append + length
    if case.bias_ids is not None:
        b += case.bias_ids.nbytes + case.bias_vals.nbytes
    if case.allowed_bits is not None:
        b += case.allowed_bits.nbytes
    for a in (case.temperature, case.top_k, case.top_p, case.min_p, case.rep_pen, case.pres_pen, case.freq_pen):
        if a is not None:
            b += a.nbytes
    b += case.B * 16 + case.B * 8  # seed + offset read, offset write
    b += case.B * 8  # ids out
    return int(b)


class ClockSampler:
    """Polls NVML (SM clock + clock-event reasons) on a thread while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int, period_s: float = 0.002):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"], "samples": 0}
        reasons = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples)}


def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if args.impl == "ours" else "gloo"
        if args.impl == "ours":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif args.impl == "ours":
        torch.cuda.set_device(0)
    return world, rank, local


def cpu_baseline(case, budget_s: float = 10.0, max_rows: int | None = None):
    """Time the oracle (C, all host cores) on whole batches of the workload."""
    from oracle import oracle

    threads = os.cpu_count() or 1
    oracle.build()
    oracle.run(case, threads=threads)  # warm
    rows = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        oracle.run(case, threads=threads)
        rows += case.B
        if max_rows and rows >= max_rows:
            break
    dt = time.perf_counter() - t0
    return {"value": rows / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{rows} rows of {case.name} ({rows // case.B} full batches) through the C oracle "
                      f"with {threads} OpenMP threads, {dt:.1f} s"}


def run_reference(args, world, rank):
    """CPU arm: the spec restatement on the host cores, rank 0 only."""
    from oracle import oracle
    from mstar_rs_b200 import workloads as W

    if rank != 0:
        return
    case = make_case(args, 0)
    threads = os.cpu_count() or 1
    oracle.build()
    t0 = time.perf_counter()
    oracle.run(case, threads=threads)
    t_batch = time.perf_counter() - t0
    budget = 90.0
    rows_per_step = case.B
    if (args.steps + args.warmup) * t_batch > budget:
        rows_per_step = max(1, int(case.B * budget / ((args.steps + args.warmup) * t_batch)))
    sub = case.row_slice(0, rows_per_step) if rows_per_step < case.B else case
    for _ in range(args.warmup):
        oracle.run(sub, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.run(sub, threads=threads)
    dt = time.perf_counter() - t0
    value = rows_per_step * args.steps / dt
    sample = (f"{args.steps} steps of {rows_per_step} rows of {case.name} through the C oracle "
              f"(spec restatement) with {threads} OpenMP threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_of(case, args, world, rows_per_step=rows_per_step),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def config_of(case, args, world, **extra):
    c = {"workload": case.name, "B": case.B, "V": case.V, "logits_dtype": case.dtype,
         "history": None if case.hist_ids is None else int(case.hist_ids.shape[1]),
         "parallelism": f"dp{world}" if world > 1 else "single",
         "rng": "philox in-kernel, offset advanced per step", "state_updates": "history append + offset",
         "history_reset": "restored from the initial Zipf history once per cycle over the logits buffers"}
    c.update(extra)
    return c


def run_ours(args, world, rank, local):
    import numpy as np
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel, workloads as W

    dev = torch.device("cuda", local)
    case = make_case(args, rank)
    d = W.to_device(case, device=dev, with_uniforms=False)
    if d.get("seed") is None:
        d["seed"] = torch.arange(case.B, dtype=torch.int64, device=dev) + 12345
        d["offset"] = torch.zeros(case.B, dtype=torch.int64, device=dev)
    base = d.pop("logits")
    step_bytes = base.numel() * base.element_size()
    nbuf = max(2, -(-2 * L2_BYTES // step_bytes))
    bufs = [base] + [torch.roll(base, shifts=997 * i, dims=1).contiguous() for i in range(1, nbuf)]
    B = case.B
    out = torch.zeros(B, dtype=torch.int64, device=dev)
    flags = N.FLAG_ADVANCE_OFFSET | (N.FLAG_UPDATE_HISTORY if d.get("hist_ids") is not None else 0)
    params = [kernel.build_params(b, **d, out_ids=out, flags=flags, cluster_size=args.cluster) for b in bufs]

    # The logits buffers repeat every nbuf steps, so tokens appended to the
    # history would pile up penalties on the same ids step after step and
    # drift the workload away from its 1024-token Zipf history; the history
    # is therefore restored (device copy, inside the timed graphs) at the
    # start of every cycle over the buffers.
    hist0 = None
    if d.get("hist_ids") is not None:
        hist0 = (d["hist_ids"].clone(), d["hist_len"].clone())

    def restore(i):
        if hist0 is not None and i % nbuf == 0:
            d["hist_ids"].copy_(hist0[0])
            d["hist_len"].copy_(hist0[1])

    def step(i):
        restore(i)
        kernel.launch_step(params[i % nbuf], dev)

    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for i in range(max(3, args.warmup)):
            step(i)
    torch.cuda.synchronize(dev)

    K = args.steps
    g = min(K, 8 * nbuf)
    reps, rem = divmod(K, g)

    def capture(n, with_events=False, start=0):
        graph = torch.cuda.CUDAGraph()
        evs = []
        with torch.cuda.graph(graph, stream=stream):
            for i in range(n):
                if with_events:
                    e0 = torch.cuda.Event(enable_timing=True, external=True)
                    e1 = torch.cuda.Event(enable_timing=True, external=True)
                    restore(start + i)
                    e0.record()
                    kernel.launch_step(params[(start + i) % nbuf], dev)
                    e1.record()
                    evs.append((e0, e1))
                else:
                    step(start + i)
        return graph, evs

    gmain, _ = capture(g)
    grem, _ = capture(rem, start=g * reps) if rem else (None, [])
    gev, evs = capture(min(g, 2 * nbuf), with_events=True)
    with torch.cuda.stream(stream):
        gmain.replay()  # graph warm-up
    torch.cuda.synchronize(dev)

    dist = None
    if world > 1:
        import torch.distributed as dist
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    with clocks:
        with torch.cuda.stream(stream):
            t0.record(stream)
            for _ in range(reps):
                gmain.replay()
            if grem is not None:
                grem.replay()
            t1.record(stream)
        torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    if dist:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())

    # kernel durations (events around each launch, cold buffers)
    with torch.cuda.stream(stream):
        gev.replay()
    torch.cuda.synchronize(dev)
    kdur = [a.elapsed_time(b) for a, b in evs]
    k_ms = statistics.mean(kdur)

    # e2e through the public API from pinned host memory
    e2e = run_e2e(args, case, d, dev, stream, world)

    if rank != 0:
        return
    rows = B * K * world
    value = rows / (ms / 1e3)
    alg = algorithmic_bytes(case)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:  # noqa: BLE001
        pass
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    # the kernel's average launch duration over the timed region (one launch
    # per step, back to back from the graph, as in a decode loop); the mean
    # of events placed around each single launch is reported beside it
    # (those events add their own overhead and keep launches from overlapping)
    region_ms = ms / K
    achieved = alg / (region_ms / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get(case.name)
        except Exception:  # noqa: BLE001
            traffic = None
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(case, args, world, l2=f"{nbuf} rotating logits buffers "
                            f"({nbuf * step_bytes / 2**20:.0f} MiB > 2x L2)",
                            launch="CUDA graph replay", cluster_size=kernel.plan(bufs[0], **d, out_ids=out)[0]),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
                     "kernel_us": region_ms * 1e3, "kernel_us_isolated": k_ms * 1e3,
                     "algorithmic_bytes": alg},
        "e2e": e2e,
        "gpu_launches": K,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(case)
    print(json.dumps(line), flush=True)


def run_e2e(args, case, d, dev, stream, world):
    """Same workload through mstar_rs_b200.sampling (the drop-in API) with the
    logits in pinned host memory: H2D copy, sample, D2H of the ids, per step."""
    import torch

    from mstar_rs_b200 import sampling

    B, V = case.B, case.V
    dt = torch.bfloat16 if case.dtype == "bf16" else torch.float32
    host = [torch.empty(B, V, dtype=dt).pin_memory() for _ in range(2)]
    src = d  # noqa: F841
    import numpy as np

    lf = case.logits_f32()
    for i, h in enumerate(host):
        h.copy_(torch.from_numpy(np.roll(lf, 13 * i, axis=1)).to(dt))
    engine = sampling.Sampler(device=dev, max_requests=max(256, B))
    rids = [f"r{i}" for i in range(B)]
    for i, rid in enumerate(rids):
        engine.add_request(rid)
        engine.set_config(rid, vocab_size=V, temperature=float(case.temperature[i]),
                          top_k=int(case.top_k[i]) if case.top_k is not None else 0,
                          top_p=float(case.top_p[i]) if case.top_p is not None else 1.0,
                          min_p=float(case.min_p[i]) if case.min_p is not None else 0.0,
                          repetition_penalty=float(case.rep_pen[i]) if case.rep_pen is not None else 1.0,
                          presence_penalty=float(case.pres_pen[i]) if case.pres_pen is not None else 0.0,
                          frequency_penalty=float(case.freq_pen[i]) if case.freq_pen is not None else 0.0)
        engine._sampling_config[rid].set_seed(1000 + i)
        if case.hist_ids is not None:
            engine.set_history(rid, case.hist_ids[i, : int(case.hist_len[i])].tolist())
    # Double-buffered: step i+1's logits cross PCIe on a copy stream while
    # step i samples; a buffer is refilled only after the step that read it.
    dev_logits = [torch.empty(B, V, dtype=dt, device=dev) for _ in range(2)]
    ids_host = [torch.empty(B, dtype=torch.int64).pin_memory() for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    n = args.e2e_steps

    def steps(count, start_ev=None):
        if start_ev is not None:
            copy_stream.wait_event(start_ev)
        for i in range(count):
            j = i % 2
            with torch.cuda.stream(copy_stream):
                if i >= 2:
                    copy_stream.wait_event(free[j])
                dev_logits[j].copy_(host[j], non_blocking=True)
                ready[j].record(copy_stream)
            with torch.cuda.stream(stream):
                stream.wait_event(ready[j])
                tok = engine.sample(rids, dev_logits[j], apply_penalty=True)
                free[j].record(stream)
                ids_host[j].copy_(tok, non_blocking=True)

    steps(3)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    steps(n, start_ev=e0)
    e1.record(stream)  # after the last step's sample and id read, which follow every copy
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist

        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    return {"value": B * n * world / (ms / 1e3), "unit": "rows/s",
            "h2d_bytes_per_step": B * V * host[0].element_size(), "d2h_bytes_per_step": B * 8,
            "steps": n, "api": "mstar_rs_b200.sampling.Sampler.sample (eager)",
            "pipeline": "two device logits buffers; step i+1's H2D copy overlaps step i's sampling"}


def run_tp(args, world, rank, local):
    """Vocab-parallel sampling (B=128, V=152064 bf16 split evenly over the
    ranks): each step is this rank's shard records, an NCCL all-gather of the
    records and the merge that gives every rank the same ids.  Strong scaling:
    the rows and the vocabulary are fixed, the ranks share the vocabulary."""
    import torch

    from mstar_rs_b200 import tp as TP
    from mstar_rs_b200 import workloads as W

    dev = torch.device("cuda", local)
    shard = W.tp_sharded(world, seed=args.seed)[rank]
    d = W.to_device(shard, device=dev)
    base = d.pop("logits")
    off = int(d.pop("vocab_offset", shard.vocab_offset) or 0)
    V_global = shard.V * world
    step_bytes = base.numel() * base.element_size()
    nbuf = max(2, -(-2 * L2_BYTES // step_bytes))
    bufs = [base] + [torch.roll(base, shifts=997 * i, dims=1).contiguous() for i in range(1, nbuf)]
    B = shard.B
    gather = None if world > 1 else (lambda recv, send: recv.copy_(send))
    smp = TP.VocabParallelSampler(B, V_global, world, rank, dev, tp_cap=64, gather=gather)
    out = torch.zeros(B, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        smp.sample(bufs[i % nbuf], off, out, **d)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize(dev)
    K = args.steps
    # One rank: the exchange is a device copy, so the whole step is captured
    # once per buffer cycle and replayed (as a decode graph would hold it).
    # More ranks: eager steps, the NCCL all-gather issued from the host.
    graphs = []
    if world == 1:
        reps, rem = divmod(K, nbuf)
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(stream)
        for n in (nbuf, rem):
            if n == 0:
                continue
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for i in range(n):
                    step(i)
            graphs.append(g)
        stream.wait_stream(cap)
        for g in graphs:  # graph warm-up (uploads the graphs)
            g.replay()
        torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    if graphs:
        for _ in range(reps):
            graphs[0].replay()
        if rem:
            graphs[-1].replay()
    else:
        for i in range(K):
            step(i)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1)
    if world > 1:
        dist.barrier()
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    if rank != 0:
        return
    print(json.dumps({
        "metric": METRIC, "value": B * K / (ms / 1e3), "unit": "rows/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"tp{world}_b{B}_v{V_global}_bf16", "B": B, "V": V_global, "logits_dtype": "bf16",
                   "history": int(shard.hist_ids.shape[1]), "parallelism": f"tp{world}",
                   "launch": ("CUDA graph replay: shard records, exchange copy, merge per step" if graphs
                              else "eager: shard records, NCCL all-gather, merge per step"),
                   "l2": f"{nbuf} rotating shard buffers ({nbuf * step_bytes / 2**20:.0f} MiB > 2x L2)"},
        "gpu_launches": 2 * K,
    }), flush=True)


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "tp":
            run_tp(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
