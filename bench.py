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
            the timed region.  e2e: the same steps through the public Python API
            from pinned host logits (H2D + step + D2H of the ids timed).
            api_graph: the drop-in CudaGraphableSampler replayed with the
            engine's stage / gather / sync around every replay, device logits.
            per_config (one GPU): every other workload the sampler is measured
            on, each with its roofline and CPU baseline.  lmhead (one GPU): the
            tensor-core LM-head projection + sampling call against cuBLAS + the
            same sampler step.
            More GPUs (torchrun): the line is data-parallel (each rank its own
            batch, weak scaling); `tp` is the vocabulary-sharded workload over
            the ranks (shard records, NCCL all-gather, merge, captured in one
            graph) and `dp_split` the constrained workload's 512 rows split
            across the ranks (strong scaling).
reference:  the torch-formulated CPU restatement of the sampler (oracle/
            torch_ref.py, batched over the rows, all host cores), rank 0 only,
            on a bounded sample of the same workload.
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
    ap.add_argument("--no-per-config", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--only", choices=["lmhead"], default=None,
                    help="print only the LM-head report (projection + sampling against cuBLAS + sampler)")
    ap.add_argument("--lmhead-profile", type=int, default=0, metavar="N",
                    help="run N plain projection + sampling calls (no graphs, no timing) for a profiler")
    return ap.parse_args()


def make_case(name, rank=0, seed=0, bucket=128):
    """The workload's batch.  Every data-parallel rank samples the same seeded
    batch (weak scaling: the per-GPU work is the one-GPU run's, row for row;
    batches drawn per rank differ in their heaviest row, e.g. one min_p row
    with 1,700 candidates, and the max over ranks would time that instead)."""
    from mstar_rs_b200 import workloads as W

    if name == "qwen_mixed":
        return W.qwen_mixed(seed=seed)
    if name == "orpheus_single":
        return W.orpheus_single(seed=seed)
    if name == "bucket":
        return W.bucket_sweep(bucket, seed=seed)
    if name == "tp":  # the whole row (the reference arm samples it unsharded)
        return W.tp_full(W.tp_sharded(1, seed=seed))
    return W.constrained(seed=seed)


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


def config_of(case, world):
    """The workload description both arms print (the same keys in both)."""
    return {"workload": case.name, "B": case.B, "V": case.V, "logits_dtype": case.dtype,
            "history": None if case.hist_ids is None else int(case.hist_ids.shape[1]),
            "parallelism": f"dp{world} (every rank samples the same seeded batch)" if world > 1 else "single",
            "rng": "philox in-kernel, offset advanced per step",
            "state_updates": "history append + offset" if case.hist_ids is not None else "offset",
            "history_reset": "restored from the initial Zipf history once per cycle over the logits buffers",
            "l2": "inputs larger than 2x L2 per step (rotating logits buffers)"}


def torch_cpu_baseline(case, budget_s: float = 8.0, max_rows: int | None = None):
    """The torch-formulated CPU sampler (oracle/torch_ref.py, batched over the
    rows, every host core) on a bounded sample of the workload's rows."""
    import torch

    from oracle import torch_ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = min(case.B, max(1, max_rows or case.B))
    sub = case.row_slice(0, rows) if rows < case.B else case
    torch_ref.run_batched(sub)  # warm
    done, t0 = 0, time.perf_counter()
    while True:
        torch_ref.run_batched(sub)
        done += rows
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{done} rows of {case.name} ({done // rows} batches of {rows}) through the torch-formulated "
                      f"CPU sampler (float64 softmax, sort, cumsum; {threads} threads), {dt:.1f} s"}


def c_oracle_baseline(case, budget_s: float = 4.0):
    """The C spec oracle (OpenMP over rows, every host core), for reference."""
    from oracle import oracle

    threads = os.cpu_count() or 1
    oracle.build()
    oracle.run(case, threads=threads)
    rows, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        oracle.run(case, threads=threads)
        rows += case.B
    return {"value": rows / (time.perf_counter() - t0), "unit": "rows/s", "cores": threads,
            "kind": "port", "sample": f"{rows} rows of {case.name} through the C spec oracle"}


def run_reference(args, world, rank):
    """CPU arm: the torch-formulated sampler on the host cores, rank 0 only,
    each step a bounded sample of the workload's rows."""
    import torch

    from oracle import torch_ref

    if rank != 0:
        return
    case = make_case(args.workload, 0, args.seed, args.bucket)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    probe = case.row_slice(0, min(case.B, 8)) if case.B > 8 else case
    torch_ref.run_batched(probe)  # the first call pays thread-pool and allocator set-up
    t0 = time.perf_counter()
    torch_ref.run_batched(probe)
    per_row = (time.perf_counter() - t0) / probe.B
    budget = 120.0
    rows_per_step = case.B
    if (args.steps + args.warmup) * per_row * case.B > budget:
        rows_per_step = max(1, int(budget / ((args.steps + args.warmup) * per_row)))
    sub = case.row_slice(0, rows_per_step) if rows_per_step < case.B else case
    for _ in range(args.warmup):
        torch_ref.run_batched(sub)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        torch_ref.run_batched(sub)
    dt = time.perf_counter() - t0
    value = rows_per_step * args.steps / dt
    sample = (f"{args.steps} steps of {rows_per_step} rows of {case.name} through the torch-formulated CPU "
              f"sampler (oracle/torch_ref.py, batched, {threads} threads)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_of(case, world),
        "rows_per_step": rows_per_step,
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _peak():
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:  # noqa: BLE001
        peaks = {}
    p = peaks.get("hbm_gbs")
    return (p, "measured") if p else (6650.0, "fallback")


def _rotating(base, torch):
    step_bytes = base.numel() * base.element_size()
    nbuf = max(2, -(-2 * L2_BYTES // step_bytes))
    return [base] + [torch.roll(base, shifts=997 * i, dims=1).contiguous() for i in range(1, nbuf)], nbuf


def time_graph_steps(case, dev, stream, steps, warmup, cluster=0, restore_history=True):
    """Graph replay of `steps` sampling steps of `case` over rotating cold
    buffers; returns (ms per step, mean isolated launch ms, cluster width)."""
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel
    from mstar_rs_b200 import workloads as W

    d = W.to_device(case, device=dev, with_uniforms=False)
    if d.get("seed") is None:
        slots = case.temperature.shape[0] if case.temperature is not None else case.B
        d["seed"] = torch.arange(slots, dtype=torch.int64, device=dev) + 12345
        d["offset"] = torch.zeros(slots, dtype=torch.int64, device=dev)
    base = d.pop("logits")
    bufs, nbuf = _rotating(base, torch)
    out = torch.zeros(case.B, dtype=torch.int64, device=dev)
    flags = N.FLAG_ADVANCE_OFFSET | (N.FLAG_UPDATE_HISTORY if d.get("hist_ids") is not None else 0)
    params = [kernel.build_params(b, **d, out_ids=out, flags=flags, cluster_size=cluster) for b in bufs]
    # The logits buffers repeat every nbuf steps, so tokens appended to the
    # history would pile up penalties on the same ids step after step; the
    # history is restored (device copy, inside the timed graphs) at the start
    # of every cycle over the buffers.
    hist0 = None
    if d.get("hist_ids") is not None and restore_history:
        hist0 = (d["hist_ids"].clone(), d["hist_len"].clone())

    def step(i):
        if hist0 is not None and i % nbuf == 0:
            d["hist_ids"].copy_(hist0[0])
            d["hist_len"].copy_(hist0[1])
        kernel.launch_step(params[i % nbuf], dev)

    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for i in range(max(3, warmup)):
            step(i)
    torch.cuda.synchronize(dev)
    g = min(steps, 8 * nbuf)
    reps, rem = divmod(steps, g)

    def capture(n, start=0, events=False):
        graph = torch.cuda.CUDAGraph()
        evs = []
        with torch.cuda.graph(graph, stream=stream):
            for i in range(n):
                if events:
                    e0 = torch.cuda.Event(enable_timing=True, external=True)
                    e1 = torch.cuda.Event(enable_timing=True, external=True)
                    e0.record()
                    step(start + i)
                    e1.record()
                    evs.append((e0, e1))
                else:
                    step(start + i)
        return graph, evs

    gmain, _ = capture(g)
    grem = capture(rem, start=g * reps)[0] if rem else None
    gev, evs = capture(min(g, 2 * nbuf), events=True)
    with torch.cuda.stream(stream):
        gmain.replay()
    torch.cuda.synchronize(dev)
    return dict(graphs=(gmain, grem, reps), events=(gev, evs), plan=kernel.plan(bufs[0], **d, out_ids=out)[0],
                step_bytes=base.numel() * base.element_size(), nbuf=nbuf)


def prewarm(t, stream, dev):
    """One untimed replay of the main graph (same work as a timed one)."""
    import torch

    with torch.cuda.stream(stream):
        t["graphs"][0].replay()
    torch.cuda.synchronize(dev)


def replay_ms(t, stream, dev):
    import torch

    gmain, grem, reps = t["graphs"]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        # one untimed replay queued first: the device is busy while the timed
        # replays are submitted, so host submission delays (several ranks
        # sharing the host's cores) stay outside the K timed steps
        gmain.replay()
        e0.record(stream)
        for _ in range(reps):
            gmain.replay()
        if grem is not None:
            grem.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1)


def isolated_ms(t, stream, dev):
    import torch

    gev, evs = t["events"]
    with torch.cuda.stream(stream):
        gev.replay()
    torch.cuda.synchronize(dev)
    return statistics.mean(a.elapsed_time(b) for a, b in evs)


def run_ours(args, world, rank, local):
    import torch

    dev = torch.device("cuda", local)
    case = make_case(args.workload, rank, args.seed, args.bucket)
    stream = torch.cuda.Stream(device=dev)
    K = args.steps
    t = time_graph_steps(case, dev, stream, K, args.warmup, cluster=args.cluster)

    dist = None
    if world > 1:
        import torch.distributed as dist
    # untimed replays for ~50 ms before the timed region, so that a short K
    # (a few hundred microseconds of work) is timed at steady clocks
    t_end = time.perf_counter() + 0.05
    while time.perf_counter() < t_end:
        prewarm(t, stream, dev)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    with clocks:
        ms = replay_ms(t, stream, dev)
    rank_us = None
    if dist:
        dist.barrier()
        tt = torch.tensor([ms], device=dev)
        every = [torch.zeros_like(tt) for _ in range(world)]
        dist.all_gather(every, tt)
        rank_us = [round(float(x.item()) * 1e3 / K, 3) for x in every]
        ms = max(float(x.item()) for x in every)
    k_ms = isolated_ms(t, stream, dev)

    e2e = run_e2e(args, case, dev, stream, world)
    api = run_api_graph(case, dev, world)
    extra = {}
    if world > 1:
        extra["tp"] = run_tp_multi(args, world, rank, local)
        extra["tp_topk_off"] = run_tp_topk_off(args, world, rank, local)
        extra["dp_split"] = run_dp_split(args, world, rank, local)
    plan, nbuf, step_bytes = t["plan"], t["nbuf"], t["step_bytes"]
    del t
    if rank != 0:
        return
    rows = case.B * K * world
    value = rows / (ms / 1e3)
    alg = algorithmic_bytes(case)
    peak, peak_src = _peak()
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
        "config": config_of(case, world),
        "measurement": {"launch": "CUDA graph replay", "cluster_size": plan,
                        "l2": f"{nbuf} rotating logits buffers ({nbuf * step_bytes / 2**20:.0f} MiB)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
                     "kernel_us": region_ms * 1e3, "kernel_us_isolated": k_ms * 1e3,
                     "algorithmic_bytes": alg},
        "e2e": e2e,
        "api_graph": api,
        "gpu_launches": K,
        "clocks": clocks.summary(),
    }
    if rank_us is not None:
        line["rank_us_per_step"] = rank_us  # the line's time is their max
    line.update(extra)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = torch_cpu_baseline(case)
        line["cpu_spec_oracle"] = c_oracle_baseline(case)
    if world == 1 and not args.no_per_config and args.workload == "qwen_mixed":
        line["per_config"] = run_per_config(args, dev, stream, no_cpu=args.no_cpu_baseline)
        line["lmhead"] = run_lmhead(dev)
    print(json.dumps(line), flush=True)


def run_per_config(args, dev, stream, no_cpu=False):
    """Every other workload at one GPU: µs per step, rows/s, roofline and the
    torch-formulated CPU baseline on a few rows."""
    import torch

    out = {}
    peak, peak_src = _peak()
    for name, bucket in (("orpheus_single", 0), ("bucket", 128), ("bucket", 512), ("constrained", 0)):
        case = make_case(name, 0, args.seed, bucket)
        steps = 200 if case.B >= 256 else 500
        t = time_graph_steps(case, dev, stream, steps, 5)
        ms = replay_ms(t, stream, dev) / steps
        alg = algorithmic_bytes(case)
        ent = {"us_per_step": ms * 1e3, "rows_per_s": case.B / (ms / 1e3), "cluster_size": t["plan"],
               "roofline": {"bound": "hbm", "achieved": alg / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                            "frac": alg / (ms / 1e3) / 1e9 / peak, "peak_source": peak_src,
                            "algorithmic_bytes": alg}}
        if not no_cpu:
            ent["cpu_baseline"] = torch_cpu_baseline(case, budget_s=3.0, max_rows=4)
        out[case.name] = ent
        del t
        torch.cuda.empty_cache()
    tp1 = run_tp_single(args, dev, stream)
    if not no_cpu:
        tp1["cpu_baseline"] = torch_cpu_baseline(make_case("tp", 0, args.seed), budget_s=3.0, max_rows=8)
    out[tp1.pop("name")] = tp1
    return out


def _graph_us(fn, dev, reps=10, replays=5):
    """Mean µs of one fn() call, fn captured `reps` times in a CUDA graph."""
    import torch

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(replays):
            g.replay()
        e1.record(s)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / (reps * replays)
    del g
    return ms * 1e3


def run_lmhead(dev, B=64, V=151936, d=2048):
    """The LM-head projection feeding the sampler (one GPU, the mixed
    workload's rows and histories, operands whose projection has the mixed
    workload's logits): the tensor-core projection + sampling call against
    cuBLAS's bf16 GEMM followed by the same sampler step.  Weights stream
    from HBM every call (V * d * 2 bytes > L2); the logits stay in L2."""
    import torch

    from mstar_rs_b200 import kernel
    from mstar_rs_b200 import workloads as W

    case = W.qwen_mixed(seed=5, B=B, V=V)
    kw = W.to_device(case, device=dev)
    kw.pop("logits")
    hidden, weight = W.lmhead_operands(B, V, d, seed=7, device=dev)
    logits = torch.empty(B, V, dtype=torch.bfloat16, device=dev)
    ids = torch.zeros(B, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    p = kernel.build_params(logits, **kw, out_ids=ids)

    def fused():
        kernel.lmhead_step(hidden, weight, logits, status=status, **kw, out_ids=ids)

    def gemm():
        kernel.lmhead_logits(hidden, weight, out=logits, status=status)

    def sampler():
        kernel.launch_step(p, dev)

    def cublas():
        torch.matmul(hidden, weight.T, out=logits)

    def cublas_then_sampler():
        cublas()
        sampler()

    r = {name: _graph_us(fn, dev) for name, fn in (("fused_us", fused), ("gemm_us", gemm),
                                                   ("sampler_l2_resident_us", sampler), ("cublas_gemm_us", cublas),
                                                   ("cublas_then_sampler_us", cublas_then_sampler))}
    torch.cuda.synchronize(dev)
    wbytes = V * d * 2
    alg = wbytes + hidden.numel() * 2 + algorithmic_bytes(case) - B * V * 2  # the logits stay on chip
    peak, peak_src = _peak()
    ach = alg / (r["fused_us"] * 1e-6) / 1e9
    out = {"config": {"B": B, "V": V, "d": d, "dtype": "bf16", "workload": "qwen_mixed rows, projected logits"},
           **{k: round(v, 2) for k, v in r.items()},
           "gemm_weights_gbs": wbytes / (r["gemm_us"] * 1e-6) / 1e9,
           "cublas_weights_gbs": wbytes / (r["cublas_gemm_us"] * 1e-6) / 1e9,
           "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                        "peak_source": peak_src, "algorithmic_bytes": alg},
           "status": int(status.item())}
    del hidden, weight, logits
    torch.cuda.empty_cache()
    return out


def run_e2e(args, case, dev, stream, world):
    """Same workload through mstar_rs_b200.sampling (the drop-in API) with the
    logits in pinned host memory: H2D copy, sample, D2H of the ids, per step."""
    import numpy as np
    import torch

    from mstar_rs_b200 import sampling

    B, V = case.B, case.V
    dt = torch.bfloat16 if case.dtype == "bf16" else torch.float32
    host = [torch.empty(B, V, dtype=dt).pin_memory() for _ in range(2)]
    lf = case.logits_f32()
    for i, h in enumerate(host):
        h.copy_(torch.from_numpy(np.roll(lf, 13 * i, axis=1)).to(dt))
    engine = sampling.Sampler(device=dev, max_requests=max(256, B))
    rids = [f"r{i}" for i in range(B)]
    _configure(engine, rids, case)
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


def _configure(engine, rids, case):
    for i, rid in enumerate(rids):
        engine.add_request(rid)
        engine.set_config(rid, vocab_size=case.V, temperature=float(case.temperature[i]),
                          top_k=int(case.top_k[i]) if case.top_k is not None else 0,
                          top_p=float(case.top_p[i]) if case.top_p is not None else 1.0,
                          min_p=float(case.min_p[i]) if case.min_p is not None else 0.0,
                          repetition_penalty=float(case.rep_pen[i]) if case.rep_pen is not None else 1.0,
                          presence_penalty=float(case.pres_pen[i]) if case.pres_pen is not None else 0.0,
                          frequency_penalty=float(case.freq_pen[i]) if case.freq_pen is not None else 0.0)
        engine._sampling_config[rid].set_seed(1000 + i)
        if case.hist_ids is not None:
            engine.set_history(rid, case.hist_ids[i, : int(case.hist_len[i])].tolist())


def run_api_graph(case, dev, world, steps=200):
    """The drop-in graph path as an engine drives it: SamplerBuffers +
    CudaGraphableSampler captured once, then per step stage / gather /
    replay / sync with device-resident logits (no host transfer)."""
    import numpy as np
    import torch

    from mstar_rs_b200 import sampling

    B, V = case.B, case.V
    dt = torch.bfloat16 if case.dtype == "bf16" else torch.float32
    sbuf = sampling.SamplerBuffers.allocate(B, dev, vocab_size=V)
    rids = [f"g{i}" for i in range(B)]
    masks = []
    for i, r in enumerate(rids):
        c = sampling.SamplingConfig(vocab_size=V, temperature=float(case.temperature[i]),
                                    top_k=int(case.top_k[i]) if case.top_k is not None else 0,
                                    top_p=float(case.top_p[i]) if case.top_p is not None else 1.0,
                                    min_p=float(case.min_p[i]) if case.min_p is not None else 0.0,
                                    repetition_penalty=float(case.rep_pen[i]) if case.rep_pen is not None else 1.0,
                                    presence_penalty=float(case.pres_pen[i]) if case.pres_pen is not None else 0.0,
                                    frequency_penalty=float(case.freq_pen[i]) if case.freq_pen is not None else 0.0)
        c.set_seed(2000 + i)
        sbuf.register_request(r, c)
        m = sampling.SeenTokenMask.new(r, V, dev)
        if case.hist_ids is not None:
            m.add_tokens(torch.from_numpy(case.hist_ids[i].astype(np.int64)).to(dev))
        masks.append(m)
    lf = case.logits_f32()
    base = torch.from_numpy(lf).to(dt).to(dev)
    bufs, nbuf = _rotating(base, torch)
    g_logits = torch.empty(B, V, dtype=dt, device=dev)
    sbuf.stage_seen_token_masks(rids, masks)
    sampler = sbuf.gather_for_request_ids(rids, B)
    out = torch.zeros(B, dtype=torch.int64, device=dev)

    def dec():
        out.copy_(sampler.sample(rids, g_logits, apply_penalty=True))

    saved = (sbuf.offset_buf.clone(), sbuf.seen_tokens.buf.clone())
    torch.cuda.synchronize(dev)
    dec()
    sbuf.offset_buf.copy_(saved[0])
    sbuf.seen_tokens.buf.copy_(saved[1])
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec()
    torch.cuda.synchronize(dev)

    def one(i):
        g_logits.copy_(bufs[i % nbuf])  # the LM head's output, written into the captured buffer
        sbuf.stage_seen_token_masks(rids, masks)
        sbuf.gather_for_request_ids(rids, B)
        graph.replay()
        sampler.sync_seen_token_masks(masks)

    for i in range(5):
        one(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for i in range(steps):
        one(i)
    host_us = (time.perf_counter() - t0) / steps * 1e6
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    # the logits copy alone (it stands in for the LM head's write)
    c0.record()
    for i in range(steps):
        g_logits.copy_(bufs[i % nbuf])
    c1.record()
    torch.cuda.synchronize(dev)
    copy_ms = c0.elapsed_time(c1) / steps
    del graph
    return {"value": B * world / ((ms - copy_ms) / 1e3), "unit": "rows/s", "us_per_step": (ms - copy_ms) * 1e3,
            "us_per_step_with_copy": ms * 1e3, "host_us_per_step": host_us,
            "api": "SamplerBuffers.stage_seen_token_masks / gather_for_request_ids, CUDA-graph replay of "
                   "CudaGraphableSampler.sample, sync_seen_token_masks; device-resident logits (the time of a "
                   "device copy standing in for the LM head's write is subtracted)"}


def _tp_setup(world, rank, dev, seed):
    import torch

    from mstar_rs_b200 import tp as TP
    from mstar_rs_b200 import workloads as W

    shard = W.tp_sharded(world, seed=seed)[rank]
    d = W.to_device(shard, device=dev)
    base = d.pop("logits")
    off = int(d.pop("vocab_offset", shard.vocab_offset) or 0)
    bufs, nbuf = _rotating(base, torch)
    return shard, d, bufs, nbuf, off


def run_tp_single(args, dev, stream):
    """Vocab-parallel sampling at one rank (B=128, V=152064 bf16): shard
    records, the exchange (a device copy) and the merge, captured in a graph."""
    import torch

    from mstar_rs_b200 import tp as TP

    shard, d, bufs, nbuf, off = _tp_setup(1, 0, dev, args.seed)
    B = shard.B
    smp = TP.VocabParallelSampler(B, shard.V, 1, 0, dev, tp_cap=64, gather=lambda recv, send: recv.copy_(send))
    out = torch.zeros(B, dtype=torch.int64, device=dev)
    K = 500
    with torch.cuda.stream(stream):
        for i in range(3):
            smp.sample(bufs[i % nbuf], off, out, **d)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(nbuf):
            smp.sample(bufs[i], off, out, **d)
    reps = max(1, K // nbuf)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / (reps * nbuf)
    peak, peak_src = _peak()
    alg = B * shard.V * 2 + shard.hist_ids.nbytes + B * 64
    del graph
    return {"name": f"tp1_b{B}_v{shard.V}_bf16", "us_per_step": ms * 1e3, "rows_per_s": B / (ms / 1e3),
            "roofline": {"bound": "hbm", "achieved": alg / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": alg / (ms / 1e3) / 1e9 / peak, "peak_source": peak_src, "algorithmic_bytes": alg},
            "launch": "CUDA graph: shard records, exchange copy, merge per step"}


def run_tp_multi(args, world, rank, local):
    """The vocabulary-sharded workload over the ranks: per step this rank's
    shard records, an NCCL all-gather of the records and the merge (every
    rank gets the same ids), the whole step captured in one CUDA graph.
    Reported: µs per step (max over ranks) and the all-gather's share."""
    import torch
    import torch.distributed as dist

    from mstar_rs_b200 import tp as TP

    dev = torch.device("cuda", local)
    shard, d, bufs, nbuf, off = _tp_setup(world, rank, dev, args.seed)
    B = shard.B
    smp = TP.VocabParallelSampler(B, shard.V * world, world, rank, dev, tp_cap=64, group=dist.group.WORLD)
    out = torch.zeros(B, dtype=torch.int64, device=dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(3):
            smp.sample(bufs[i % nbuf], off, out, **d)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(nbuf):
            smp.sample(bufs[i], off, out, **d)
    send = smp.send[: B * smp.words]
    recv = smp.recv[: world * B * smp.words]
    ag = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ag, stream=stream):
        for i in range(nbuf):
            dist.all_gather_into_tensor(recv, send)
    reps = max(1, 400 // nbuf)

    def timed(g):
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / (reps * nbuf)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = timed(graph)
    ag_ms = timed(ag)
    ids_ok = torch.tensor([1], device=dev)
    ref = out.clone()
    dist.broadcast(ref, src=0)
    ids_ok[0] = int(torch.equal(ref, out))
    dist.all_reduce(ids_ok, op=dist.ReduceOp.MIN)
    del graph, ag
    return {"workload": f"tp{world}_b{B}_v{shard.V * world}_bf16", "us_per_step": ms * 1e3,
            "rows_per_s": B / (ms / 1e3), "allgather_us": ag_ms * 1e3, "allgather_share": ag_ms / ms,
            "record_bytes_per_rank": B * smp.words * 4, "ids_identical_on_every_rank": bool(ids_ok.item()),
            "scaling": "strong", "launch": "one CUDA graph per cycle: tp_local, NCCL all-gather, tp_merge"}


def run_tp_topk_off(args, world, rank, local, B=128, V=152064):
    """Rows without top_k over the ranks (two rounds: records, NCCL
    all-gather, first merge, exact shard masses, a second 8-byte-per-row
    all-gather, second merge), the whole step captured in one CUDA graph.
    Reported: µs per step (max over ranks), the rows the two rounds decided,
    and whether every rank drew the same ids."""
    import torch
    import torch.distributed as dist

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import tp as TP
    from mstar_rs_b200 import workloads as W

    dev = torch.device("cuda", local)
    shard = W.tp_topk_off(world, seed=args.seed, B=B, V=V, H=512)[rank]
    d = W.to_device(shard, device=dev)
    logits = d.pop("logits")
    off = d.pop("vocab_offset")
    smp = TP.VocabParallelSampler(B, V, world, rank, dev, group=dist.group.WORLD, two_round=True, V_shard=shard.V)
    out = torch.zeros(B, dtype=torch.int64, device=dev)
    st = torch.zeros(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            smp.sample(logits, off, out, out_status=st, **d)
    torch.cuda.synchronize(dev)
    reps = 20
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(reps):
            smp.sample(logits, off, out, out_status=st, **d)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(5):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / (5 * reps)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    decided = int(((st & N.STATUS_TP_OVERFLOW) == 0).sum().item())
    ref = out.clone()
    dist.broadcast(ref, src=0)
    ok = torch.tensor([int(torch.equal(ref, out))], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    del graph
    return {"workload": f"tp{world}_topk_off_b{B}_v{V}_bf16", "us_per_step": ms * 1e3, "rows_per_s": B / (ms / 1e3),
            "rows_decided": decided, "rows": B, "ids_identical_on_every_rank": bool(ok.item()), "scaling": "strong",
            "launch": "one CUDA graph: tp_local2, all-gather, tp_merge1, tp_mass, all-gather, tp_merge2"}


def run_dp_split(args, world, rank, local):
    """The constrained workload's 512 rows split evenly across the ranks (no
    collective on the data path); µs per step is the max over ranks."""
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local)
    full = make_case("constrained", 0, args.seed)
    per = full.B // world
    case = full.row_slice(rank * per, (rank + 1) * per)
    case.name = f"constrained_b{full.B}_split{world}"
    stream = torch.cuda.Stream(device=dev)
    t = time_graph_steps(case, dev, stream, 100, 5)
    dist.barrier()
    ms = replay_ms(t, stream, dev) / 100
    tt = torch.tensor([ms], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    del t
    return {"workload": case.name, "rows_per_rank": per, "us_per_step": ms * 1e3, "rows_per_s": full.B / (ms / 1e3),
            "scaling": "strong"}


def run_tp_line(args, world, rank, local):
    """--workload tp: the vocabulary-sharded workload as the line itself
    (strong scaling over the ranks)."""
    import torch

    dev = torch.device("cuda", local)
    if world == 1:
        r = run_tp_single(args, dev, torch.cuda.Stream(device=dev))
        r["workload"] = r.pop("name")
    else:
        r = run_tp_multi(args, world, rank, local)
    if rank != 0:
        return
    case = make_case("tp", 0, args.seed)
    print(json.dumps({
        "metric": "vocab-parallel sampled rows/sec at B=128, V=152064 bf16", "value": r["rows_per_s"],
        "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["us_per_step"] / 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(config_of(case, world), workload=r["workload"], parallelism=f"tp{world}"), "tp": r,
        "gpu_launches": 2,
    }), flush=True)


def lmhead_profile(n, B=64, V=151936, d=2048):
    """n plain projection + sampling calls of the LM-head report's workload,
    one launch pair each, for ncu launch lists and captures."""
    import torch

    from mstar_rs_b200 import kernel
    from mstar_rs_b200 import workloads as W

    dev = torch.device("cuda", 0)
    case = W.qwen_mixed(seed=5, B=B, V=V)
    kw = W.to_device(case, device=dev)
    kw.pop("logits")
    hidden, weight = W.lmhead_operands(B, V, d, seed=7, device=dev)
    logits = torch.empty(B, V, dtype=torch.bfloat16, device=dev)
    ids = torch.zeros(B, dtype=torch.int64, device=dev)
    for _ in range(n):
        kernel.lmhead_step(hidden, weight, logits, **kw, out_ids=ids)
    torch.cuda.synchronize(dev)
    print(json.dumps({"lmhead_profile_calls": n, "ids": ids[:8].tolist()}))


def main():
    args = parse()
    if args.lmhead_profile:
        lmhead_profile(args.lmhead_profile)
        return
    if args.only == "lmhead":
        import torch

        print(json.dumps(run_lmhead(torch.device("cuda", 0))), flush=True)
        return
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "tp":
            run_tp_line(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
