#!/usr/bin/env python3
"""Benchmark of the TriAttention eviction step (score -> select -> compact).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME]
                    [--impl ours|reference] [--scaling weak|strong]

One step = one tria_evict call over the whole cache (every (layer, kv-head)
of the workload): score every row, select the rows to keep, compact K/V and
positions into the ping-pong buffer.  Inputs are resident in HBM and larger
than L2 (no flush needed).  Prints one JSON line on rank 0.

Under torchrun (N > 1) every rank runs its own shard:
  --scaling strong (default for N > 1) the workload's layers are partitioned
                   into contiguous blocks, one per rank (36 layers over 8
                   ranks: 5,5,5,5,4,4,4,4); total work fixed, no collective
                   on the data path;
  --scaling weak   each rank evicts a full cache of the workload (per-GPU
                   work fixed; e.g. one sequence per GPU).
The step is timed on the device with CUDA events and reported as the max over
ranks.  `--impl reference` times the reference's CPU implementation
(oracle/_ref = the reference's triattention.c, plus the oracle's select and
compact) on the host cores with all threads, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import tempfile
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "triattention-ggml_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

import numpy as np  # noqa: E402

import workloads  # noqa: E402

METRIC = "KV rows scored+evicted+compacted per sec"
UNIT = "rows/s"
FALLBACK_HBM_GBS = 6650.0

CONFIGS = {
    # Qwen3-8B geometry, the north-star step
    "qwen3-8b-f16-32k": dict(L=36, H=32, KV=8, hd=128, n=32768, type=workloads.TYPE_F16,
                             budget_pct=12, ramp=100, theta=1e6),
    # 27B-class geometry (64 layers, gqa 5)
    "27b-f16-64k": dict(L=64, H=40, KV=8, hd=128, n=65536, type=workloads.TYPE_F16,
                        budget_pct=12, ramp=100, theta=1e6),
    # q8_0 cache, 65536 rows, one eviction at a 512-row budget (last ramp stage)
    "qwen3-8b-q8_0-64k": dict(L=36, H=32, KV=8, hd=128, n=65536, type=workloads.TYPE_Q8_0,
                              budget=512, ramp=100, theta=1e6),
    # multi-sequence server batch: 8 sequences of up to 16384 rows in one q8_0
    # cache, n_kv ~ U[8192, 16384] per sequence, a global budget of 512 rows per
    # (layer, kv-head) on average per sequence, shared across its units
    "multiseq-q8_0-global": dict(L=36, H=32, KV=8, hd=128, n=16384, type=workloads.TYPE_Q8_0,
                                 budget=512, ramp=100, theta=1e6, seqs=8),
}
DEFAULT_CONFIG = "qwen3-8b-f16-32k"
RAMP_PCTS = (10, 20, 40, 80, 100)      # the exponential ramp of one eviction schedule
RAMP_APPEND = 128                      # rows decoded between two evictions


def describe(cfg_name, c, budget):
    t = "f16" if c["type"] == workloads.TYPE_F16 else "q8_0"
    return (f"{cfg_name}: {c['L']} layers x {c['KV']} kv heads x {c['n']} rows, head_dim {c['hd']}, "
            f"gqa {c['H'] // c['KV']}, {t} K/V, budget {budget} rows per (layer, kv-head), ramp {c['ramp']}%")


def budget_rows(c):
    return int(c["n"] * c["budget_pct"] / 100) if "budget_pct" in c else int(c["budget"])


def step_bytes(c, units, keep):
    """Algorithmic bytes per step: n*Rb (K read) + 4*B*Rb (kept K, V read + write)
    + 4*n (positions read) + 8*B (positions moved), summed over units."""
    rb = workloads.row_bytes(c["type"], c["hd"])
    n = c["n"]
    return units * (n * rb + 4 * keep * rb + 4 * n + 8 * keep)


def score_kernel_bytes(c, units, layers):
    """Algorithmic bytes of one scoring launch over `units` (layer, kv-head)
    units of n rows, the scoring share of the step's bytes: every K row read
    once (n*Rb per unit) and its position (4*n per unit).  The raw scores it
    writes and the delta-table rows it reads are intermediates of the step."""
    rb = workloads.row_bytes(c["type"], c["hd"])
    n = c["n"]
    return units * (n * rb + 4 * n)


def score_kernel_traffic_bytes(c, units, layers):
    """What the scoring launch must move at least, intermediates included:
    every K row once, the shared position row once per layer, the delta table
    rows once (n rows of fc*8 bytes), and the G raw scores of every row
    written (the figure ncu's DRAM traffic is compared with)."""
    rb = workloads.row_bytes(c["type"], c["hd"])
    n, G, fc = c["n"], c["H"] // c["KV"], c["hd"] // 2
    return units * n * rb + layers * n * 4 + n * fc * 8 + units * G * n * 4


def score_kernel_flops(c, units):
    """fp32 FLOPs of the scoring math per launch: per row and frequency pair
    X, Y and |k|^2 (9 flops), then 3 FMAs (6 flops) per query head."""
    G, fc = c["H"] // c["KV"], c["hd"] // 2
    return units * c["n"] * fc * (9 + 6 * G)


def measured_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel, workload):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, or None."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)[workload][kernel]["dram_bytes_per_launch"]
    except Exception:
        return None


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) in a thread."""
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, torch_device_index, period=0.02):
        self.ok = False
        self.samples = []
        self.max_mhz = None
        try:
            import pynvml as N
            import torch
            N.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device_index).uuid)
            self.h = N.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.N = N
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - depends on the box
            self.err = repr(e)
        self.period = period
        self._stop = threading.Event()

    def _run(self):
        N = self.N
        while not self._stop.is_set():
            try:
                mhz = N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)
                rs = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": getattr(self, "err", "no samples")}
        mhz = [m for m, _ in self.samples]
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": float(statistics.median(mhz)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ---------------------------------------------------------------- CPU baseline

def cpu_data(c, n_units, seed=0):
    """Seeded K and V caches (numpy, the bench distributions) covering n_units units."""
    n_layer = max(1, (n_units + c["KV"] - 1) // c["KV"])
    if c["type"] == workloads.TYPE_F16:
        return (workloads.f16_cache(n_layer, c["n"], c["KV"], c["hd"], seed=seed),
                workloads.f16_cache(n_layer, c["n"], c["KV"], c["hd"], seed=seed + 1))
    return (workloads.q8_0_cache(n_layer, c["n"], c["KV"], c["hd"], seed=seed),
            workloads.q8_0_cache(n_layer, c["n"], c["KV"], c["hd"], seed=seed + 1))


def cpu_step_rate(c, stats_path, n_units, seed=0, threads=None, data=None, rows=None):
    """Run the reference CPU step (reference tria_score_kv_head + oracle select and
    compact, pthreads over units) on n_units units of the workload, each on its
    first `rows` rows (all of them by default; a shorter prefix keeps the same
    kept fraction).  Returns (rows/s, seconds, threads, kind)."""
    import oracle_py
    orc = oracle_py.Oracle()
    if oracle_py.RefLib.available():
        ref = oracle_py.RefLib()
        load, free, fn, kind = ref.load, ref.free, ref.score_fn_ptr, "reference"
    else:
        load, free, fn, kind = orc.load, orc.free, orc.score_fn_ptr, "port"
    threads = threads or len(os.sched_getaffinity(0))
    hd, KV, n_all = c["hd"], c["KV"], c["n"]
    n = n_all if rows is None else min(int(rows), n_all)
    rb = workloads.row_bytes(c["type"], hd)
    K, V = data if data is not None else cpu_data(c, n_units, seed)
    Ko, Vo = np.zeros_like(K), np.zeros_like(V)
    pos = np.arange(n_all, dtype=np.int32)
    pos_o = np.zeros((n_units, n_all), np.int32)
    keep = workloads.layer_keep(n, max(1, budget_rows(c) * n // n_all), c["ramp"])
    st = load(stats_path)
    units = []
    for u in range(n_units):
        l, h = divmod(u, KV)
        units.append(oracle_py.OracleUnit(l, h, n, keep, K[l, :, h * rb:].ctypes.data,
                                          V[l, :, h * rb:].ctypes.data, Ko[l, :, h * rb:].ctypes.data,
                                          Vo[l, :, h * rb:].ctypes.data, pos.ctypes.data,
                                          pos_o[u].ctypes.data, 0))
    t0 = time.perf_counter()
    rc = orc.cpu_step(fn, st, c["type"], hd, KV * rb, units, n, 0, 0, threads)
    dt = time.perf_counter() - t0
    free(st)
    assert rc == 0
    return n_units * n / dt, dt, threads, kind


def write_stats(c, td):
    path = os.path.join(td, "bench.tria")
    workloads.write_tria(path, c["L"], c["H"], c["KV"], c["hd"], rope_theta=c["theta"], seed=0)
    return path


REF_RUN_S = 90.0     # wall-time budget of a whole --impl reference run


def run_reference(args):
    """--impl reference: the reference's CPU path on the host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c = CONFIGS[args.config]
    threads = len(os.sched_getaffinity(0))
    with tempfile.TemporaryDirectory() as td:
        path = write_stats(c, td)
        # The whole run (warm-up and timed steps) is held to about REF_RUN_S
        # seconds: a step is a bounded sample of the workload.  One unit per
        # thread is timed first; a step is a whole number of such rounds when
        # that fits, else one unit per thread on a prefix of its rows.
        n_probe = min(threads, c["L"] * c["KV"])
        data = cpu_data(c, n_probe, seed=1)
        _, dt1, _, _ = cpu_step_rate(c, path, n_probe, threads=threads, data=data)
        per_step = max(0.05, min(4.0, REF_RUN_S / max(1, args.warmup + args.steps)))
        rounds = int(max(1, per_step // dt1))
        units = min(c["L"] * c["KV"], n_probe * rounds)
        if units > n_probe:
            data = cpu_data(c, units, seed=1)
        rows = c["n"] if per_step >= dt1 else max(1024, int(c["n"] * per_step / dt1) // 256 * 256)
        rates = []
        kind = "reference"
        for i in range(args.warmup + args.steps):
            r, dt, th, kind = cpu_step_rate(c, path, units, threads=threads, data=data, rows=rows)
            if i >= args.warmup:
                rates.append((r, dt))
    value = statistics.median(r for r, _ in rates)
    ms = statistics.median(dt for _, dt in rates) * 1e3
    sample = (f"{units} of {c['L'] * c['KV']} (layer, kv-head) units x {rows} of {c['n']} rows per step "
              f"(the same seeded data every step; run held to ~{REF_RUN_S:.0f} s)")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy, same distributions)",
            "config": {"workload": describe(args.config, c, budget_rows(c))},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    import devcache
    import tria_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    c = CONFIGS[args.config]
    budget = budget_rows(c)

    # shard: weak = a full workload cache per rank; strong = contiguous layer blocks
    n_head_kv, head0 = c["KV"], 0
    layer0, L = 0, c["L"]
    if args.scaling == "strong" and world > 1:
        layer0 = c["L"] * rank // world
        L = c["L"] * (rank + 1) // world - layer0
    n = c["n"]
    units = L * n_head_kv

    td = tempfile.mkdtemp()
    stats_path = write_stats(c, td)
    st = tria_b200.load(stats_path)
    ctx = tria_b200.Context(st, dev.index)
    src = devcache.DeviceCache(c["type"], L, n_head_kv, c["hd"], n, dev, layer0=layer0, head0=head0)
    dst = devcache.DeviceCache(c["type"], L, n_head_kv, c["hd"], n, dev, layer0=layer0, head0=head0)
    src.fill_synthetic(seed=1000 + rank)
    n_rows = np.full(units, n, np.int32)
    params = tria_b200.EvictParams(n, budget, c["ramp"], 0, 0, 0)
    sv, dv = src.view(shared_pos=True), dst.view()
    stream = torch.cuda.Stream(device=dev)
    keep = workloads.layer_keep(n, budget, c["ramp"])

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(dev.index)
    with clocks:
        with torch.cuda.stream(stream):
            t_w = time.perf_counter()
            i = 0
            while i < args.warmup or time.perf_counter() - t_w < 0.3:
                ctx.evict(sv, dv, n_rows, params, stream=stream)
                i += 1
                if i % 8 == 0:
                    stream.synchronize()
            stream.synchronize()
            r, counts = ctx.get_n_kv(units)
            assert (counts == keep).all(), (counts[:8], keep)

            # the step as a CUDA graph: captured once (the eager warm-up sized
            # the scratch and set the kernels' attributes), replayed per step;
            # its kernels are the eager step's, counted from one eager call
            l0 = ctx.launches()
            ctx.evict(sv, dv, n_rows, params, stream=stream)
            per_step = ctx.launches() - l0
            step_fn = lambda: ctx.evict(sv, dv, n_rows, params, stream=stream)   # noqa: E731
            graph, launch_mode = None, "eager tria_evict calls"
            if not args.no_graph:
                try:
                    graph = torch.cuda.CUDAGraph()
                    # thread-local: other threads (NCCL's watchdog) keep working during the capture
                    with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
                        ctx.evict(sv, dv, n_rows, params, stream=stream)
                    step_fn = graph.replay
                    launch_mode = "tria_evict captured once in a CUDA graph, replayed each step"
                except Exception as e:                  # noqa: BLE001 - time eager calls instead
                    graph = None
                    launch_mode = f"eager tria_evict calls (graph capture failed: {type(e).__name__})"
                    torch.cuda.synchronize()
                for _ in range(max(3, args.warmup)):
                    step_fn()
                stream.synchronize()
                r, counts = ctx.get_n_kv(units)
                assert (counts == keep).all(), (counts[:8], keep)

            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                step_fn()
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
            launches = per_step * args.steps
            ms = e0.elapsed_time(e1) / args.steps
            del graph
    clk = clocks.summary()
    ms_max = max_over_ranks(ms)

    # stage timing (CUDA events between stages, same workload).  Two steps are
    # queued back to back and the second one's events are read: reading them
    # waits for the step, so a step queued after a read would start on an
    # idle GPU and its first stages would include the host's launch time.
    ctx.set_timing(True)
    acc = {}
    with torch.cuda.stream(stream):
        for _ in range(max(3, min(args.steps, 50))):
            ctx.evict(sv, dv, n_rows, params, stream=stream)
            ctx.evict(sv, dv, n_rows, params, stream=stream)
            for k, v in ctx.stage_ms().items():
                acc.setdefault(k, []).append(v)
    ctx.set_timing(False)
    stage = {k: statistics.median(v) for k, v in acc.items()}

    # end to end through the C ABI with host buffers: the cache lives in pinned
    # host memory and tria_evict_host runs the step on it every step: K crosses
    # PCIe (staged in layer chunks against the scoring), V only for kept rows,
    # and the kept K, V and positions land in host memory; counts come back
    # through tria_get_n_kv
    e2e = None
    if not args.no_e2e:
        hk = torch.empty(src.k.shape, dtype=torch.uint8, pin_memory=True)
        hv = torch.empty(src.v.shape, dtype=torch.uint8, pin_memory=True)
        hp = torch.empty((n,), dtype=torch.int32, pin_memory=True)
        hk.copy_(src.k)
        hv.copy_(src.v)
        hp.copy_(src.pos_shared)
        ok_k = torch.empty((L, keep, src.k.shape[2]), dtype=torch.uint8, pin_memory=True)
        ok_v = torch.empty_like(ok_k, pin_memory=True)
        ok_p = torch.empty((L, n_head_kv, keep), dtype=torch.int32, pin_memory=True)
        rb = src.rb
        hsv = tria_b200.make_view(c["type"], [hk[l] for l in range(L)], [hv[l] for l in range(L)], hp, n,
                                  n_head_kv * rb, rb, n_head_kv, layer0, head0, pos_shared=True)
        hdv = tria_b200.make_view(c["type"], [ok_k[l] for l in range(L)], [ok_v[l] for l in range(L)], ok_p, keep,
                                  n_head_kv * rb, rb, n_head_kv, layer0, head0)
        h2d = units * n * rb + n * 4 + units * keep * rb
        d2h = units * keep * (2 * rb + 4) + units * 4
        e2e_steps = max(2, min(args.steps, 10))

        def e2e_step():
            ctx.evict_host(hsv, hdv, n_rows, params, stream=stream)
            return ctx.get_n_kv(units)

        with torch.cuda.stream(stream):
            _, cnt = e2e_step()
            assert (cnt == keep).all()
            stream.synchronize()
            barrier()
            t0 = time.perf_counter()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(e2e_steps):
                e2e_step()
            f1.record(stream)
            stream.synchronize()
            wall = (time.perf_counter() - t0) / e2e_steps
            dev_ms = f0.elapsed_time(f1) / e2e_steps
            barrier()
        e2e_ms = max_over_ranks(max(wall * 1e3, dev_ms))
        e2e_units = c["L"] * n_head_kv if (args.scaling == "strong" and world > 1) else units * world
        e2e = {"value": e2e_units * n / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "path": "tria_evict_host on a cache in pinned host memory: K staged to the device in layer "
                       "chunks, V read for kept rows only, kept rows written to host, counts read back"}
        del hsv, hdv, hk, hv, hp, ok_k, ok_v, ok_p

    ctx.close()
    tria_b200.free(st)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    total_units = c["L"] * n_head_kv if (args.scaling == "strong" and world > 1) else units * world
    value = total_units * n / (ms_max / 1e3)
    peak, peak_src = measured_peak()
    sb = score_kernel_bytes(c, units, L)
    score_ms = stage.get("score")
    achieved = sb / (score_ms / 1e3) / 1e9 if score_ms else None
    wl = args.config
    traffic = ncu_traffic("k_score_ws", wl)
    flops = score_kernel_flops(c, units)
    step_b = step_bytes(c, units, keep)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": args.scaling if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f32" if c["type"] == workloads.TYPE_F16 else "f32 (q8_0 cache)",
        "data": "synthetic (seeded device fill: N(0,1), 1% outlier dims x8; seeded TRIA v2 stats)",
        "config": {"workload": describe(args.config, c, budget), "layers": L, "kv_heads": c["KV"],
                   "heads": c["H"], "head_dim": c["hd"], "rows": n, "kept": keep,
                   "shard": (f"layers {layer0}..{layer0 + L - 1} of {c['L']} on rank 0 (contiguous blocks)"
                             if args.scaling == "strong" and world > 1 else f"{c['L']} layers x {n_head_kv} kv heads per rank"),
                   "l2": "inputs larger than L2 (no flush)",
                   "launch": launch_mode},
        "roofline": {"bound": "hbm", "kernel": "k_score_ws", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": (achieved / peak) if achieved else None,
                     "traffic": traffic, "peak_source": f"{peak_src} hbm_gbs",
                     "algorithmic_bytes_per_launch": sb, "launch_ms": score_ms,
                     "bytes_with_intermediates_per_launch": score_kernel_traffic_bytes(c, units, L),
                     "fp32_flops_per_launch": flops,
                     "fp32_tflops": flops / (score_ms / 1e3) / 1e12 if score_ms else None},
        "step_roofline": {"bytes_per_step": step_b, "achieved": step_b / (ms / 1e3) / 1e9,
                          "frac": step_b / (ms / 1e3) / 1e9 / peak, "unit": "GB/s"},
        "stage_ms": stage,
        "clocks": clk,
        "gpu_launches": int(launches),
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu:
        try:
            threads = len(os.sched_getaffinity(0))
            n_s = min(units, max(1, threads))
            rate, dt, th, kind = cpu_step_rate(c, stats_path, n_s, seed=7, threads=threads)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": th, "kind": kind,
                                    "sample": f"{n_s} (layer, kv-head) units x {n} rows of the same "
                                              f"workload (seeded numpy data), {dt:.1f} s wall"}
        except Exception as e:  # pragma: no cover
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "error": repr(e)}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_ramp(args):
    """--ramp-sequence: the exponential ramp of one eviction schedule.  Five
    consecutive evictions at 10/20/40/80/100 % of the way to the budget, with
    RAMP_APPEND rows decoded (appended after each unit's kept rows) between
    steps.  The five step inputs are built once by running the schedule; each
    timed step then evicts its snapshot into a scratch cache, so every step is
    the real state of the schedule and the inputs stay resident in HBM."""
    import torch
    import torch.distributed as dist

    import devcache
    import tria_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    c = CONFIGS[args.config]
    budget = budget_rows(c)
    L, KV, hd, n0 = c["L"], c["KV"], c["hd"], c["n"]
    units = L * KV
    cap = n0 + len(RAMP_PCTS) * RAMP_APPEND
    td = tempfile.mkdtemp()
    st = tria_b200.load(write_stats(c, td))
    ctx = tria_b200.Context(st, dev.index)
    stream = torch.cuda.Stream(device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(4000 + rank)

    def new_rows(n_new):
        x = torch.randn((L, n_new, KV, hd), generator=g, device=dev, dtype=torch.float32)
        if c["type"] == workloads.TYPE_F16:
            return x.half().view(torch.uint8).reshape(L, n_new, -1)
        return devcache.quantize_q8_0_torch(x).reshape(L, n_new, -1)

    snaps, rows, params = [], [], []
    s0 = devcache.DeviceCache(c["type"], L, KV, hd, cap, dev)
    s0.fill_synthetic(seed=1000 + rank, n_rows=n0)
    cur, n_rows = n0, np.full(units, n0, np.int32)
    src = s0
    with torch.cuda.stream(stream):
        for t, ramp in enumerate(RAMP_PCTS):
            snaps.append(src)
            rows.append(n_rows.copy())
            params.append(tria_b200.EvictParams(cur, budget, ramp, 0, 0, 0))
            if t == len(RAMP_PCTS) - 1:
                break
            dst = devcache.DeviceCache(c["type"], L, KV, hd, cap, dev)
            ctx.evict(src.view(shared_pos=(t == 0)), dst.view(), n_rows, params[-1], stream=stream)
            _, counts = ctx.get_n_kv(units)
            kk, vv = new_rows(RAMP_APPEND), new_rows(RAMP_APPEND)
            newpos = torch.arange(cur, cur + RAMP_APPEND, dtype=torch.int32, device=dev)
            for l in range(L):
                m = int(counts[l * KV])
                assert (counts[l * KV:(l + 1) * KV] == m).all()
                dst.k[l, m:m + RAMP_APPEND] = kk[l]
                dst.v[l, m:m + RAMP_APPEND] = vv[l]
                dst.pos[l, :, m:m + RAMP_APPEND] = newpos
            n_rows = counts.astype(np.int32) + RAMP_APPEND
            cur += RAMP_APPEND
            src = dst
        stream.synchronize()
    scratch = devcache.DeviceCache(c["type"], L, KV, hd, cap, dev)
    views = [sn.view(shared_pos=(t == 0)) for t, sn in enumerate(snaps)]
    dv = scratch.view()
    T = len(RAMP_PCTS)

    def step(i):
        t = i % T
        ctx.evict(views[t], dv, rows[t], params[t], stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()

    clocks = ClockSampler(dev.index)
    with clocks:
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                step(i)
            stream.synchronize()
            barrier()
            torch.cuda.synchronize()
            l0 = ctx.launches()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(args.steps):
                step(i)
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
            launches = ctx.launches() - l0
            ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.summary()
    if world > 1:
        t_ = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        ms = float(t_.item())
    rows_timed = sum(int(rows[i % T].sum()) for i in range(args.steps)) * world

    # per-step stage times and bytes
    ctx.set_timing(True)
    per_step = []
    with torch.cuda.stream(stream):
        for t in range(T):
            acc = {}
            for _ in range(5):
                step(t)                 # queued ahead: the timed step below starts on a busy GPU
                step(t)
                for k, v in ctx.stage_ms().items():
                    acc.setdefault(k, []).append(v)
            per_step.append({k: statistics.median(v) for k, v in acc.items()})
    ctx.set_timing(False)
    _, counts = ctx.get_n_kv(units)
    ctx.close()
    tria_b200.free(st)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    rb = workloads.row_bytes(c["type"], hd)
    keeps = [int(workloads.layer_keep(int(r[0]), budget, p.ramp_pct)) for r, p in zip(rows, params)]
    step_b = [int(r.sum()) * rb + 4 * units * k * rb + 4 * int(r.sum()) + 8 * units * k for r, k in zip(rows, keeps)]
    step_ms = [sum(v for kk, v in d.items() if kk != "table") for d in per_step]
    # the scoring share of each step's algorithmic bytes: K rows and their positions
    score_b = [int(r.sum()) * (rb + 4) for r in rows]
    score_ms = [d["score"] for d in per_step]
    peak, peak_src = measured_peak()
    ach = sum(score_b) / (sum(score_ms) / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": rows_timed / (ms * args.steps / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (q8_0 cache)" if c["type"] == workloads.TYPE_Q8_0 else "f32",
        "data": "synthetic (seeded device fill: N(0,1); seeded TRIA v2 stats; appended rows N(0,1))",
        "config": {"workload": describe(args.config, c, budget) + f"; ramp {'/'.join(map(str, RAMP_PCTS))}% "
                   f"over {T} consecutive steps, +{RAMP_APPEND} rows between steps",
                   "rows_per_step": [int(r[0]) for r in rows], "kept_per_step": keeps,
                   "l2": "inputs larger than L2 (no flush)"},
        "roofline": {"bound": "hbm", "kernel": "k_score_ws", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak, "traffic": None, "peak_source": f"{peak_src} hbm_gbs",
                     "algorithmic_bytes_per_launch": score_b, "launch_ms": score_ms},
        "step_roofline": {"bytes_per_step": step_b, "ms_per_step": step_ms,
                          "achieved": sum(step_b) / (sum(step_ms) / 1e3) / 1e9,
                          "frac": sum(step_b) / (sum(step_ms) / 1e3) / 1e9 / peak, "unit": "GB/s"},
        "stage_ms_per_step": per_step,
        "clocks": clk,
        "gpu_launches": int(launches),
        "e2e": None,
        "e2e_note": "the ramp schedule's inputs are device-resident snapshots (5 GB each); "
                    "the host-buffer path is measured on the single-step configs",
    }
    if not args.no_cpu:
        try:
            threads = len(os.sched_getaffinity(0))
            n_s = min(units, max(1, threads))
            cc = dict(c, ramp=RAMP_PCTS[0])
            rate, dt, th, kind = cpu_step_rate(cc, write_stats(c, td), n_s, seed=7, threads=threads)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": th, "kind": kind,
                                    "sample": f"{n_s} (layer, kv-head) units x {n0} rows, the first step "
                                              f"of the schedule ({RAMP_PCTS[0]}%), {dt:.1f} s wall"}
        except Exception as e:  # pragma: no cover
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "error": repr(e)}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_global(args):
    """Multi-sequence step with one global budget per sequence: every sequence's
    units are scored, the ranks (contiguous layer blocks) agree on each
    sequence's threshold key through all-gathers of key histograms (NCCL at
    N > 1), and each unit keeps its rows above it before compaction."""
    import torch
    import torch.distributed as dist

    import devcache
    import global_budget as gbud
    import tria_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    c = CONFIGS[args.config]
    n_seq, cells, KV, hd = c["seqs"], c["n"], c["KV"], c["hd"]
    layer0 = c["L"] * rank // world
    L = c["L"] * (rank + 1) // world - layer0
    units = L * KV
    rng = np.random.default_rng(77)                     # same lengths on every rank
    n_kv = rng.integers(cells // 2, cells + 1, n_seq).astype(np.int32)
    k_total = [c["budget"] * c["L"] * KV for _ in range(n_seq)]
    td = tempfile.mkdtemp()
    st = tria_b200.load(write_stats(c, td))
    ctx = tria_b200.Context(st, dev.index)
    stream = torch.cuda.Stream(device=dev)
    src = devcache.DeviceCache(c["type"], L, KV, hd, cells * n_seq, dev, layer0=layer0)
    src.fill_synthetic(seed=900 + rank)
    src.pos_shared = torch.arange(cells, dtype=torch.int32, device=dev).repeat(n_seq)
    rb = src.rb
    views, dsts, dviews, seqs, n_rows = [], [], [], [], []
    for q in range(n_seq):
        sl = slice(q * cells, (q + 1) * cells)
        views.append(tria_b200.make_view(c["type"], [src.k[l][sl] for l in range(L)], [src.v[l][sl] for l in range(L)],
                                         src.pos_shared[sl], cells, KV * rb, rb, KV, layer0, 0, pos_shared=True))
        d = devcache.DeviceCache(c["type"], L, KV, hd, cells, dev, layer0=layer0)
        dsts.append(d)
        dviews.append(d.view())
        nr = np.full(units, n_kv[q], np.int32)
        n_rows.append(nr)
        seqs.append({"scores": torch.empty((units, cells), dtype=torch.float32, device=dev), "stride": cells,
                     "n_rows": nr, "kept_idx": torch.empty((units, cells), dtype=torch.int32, device=dev),
                     "kept_stride": cells, "n_kept": torch.empty(units, dtype=torch.int32, device=dev)})

    def gather(t):
        if world == 1:
            return t[None]
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t.contiguous())
        return torch.stack(out)

    backend = gbud.DeviceBackend(dev, stream)
    one = args.global_protocol == "candidates"
    select = gbud.global_select_candidates if one else gbud.global_select

    def step():
        for q in range(n_seq):
            ctx.score(views[q], n_rows[q], int(n_kv[q]), seqs[q]["scores"], stream=stream)
        select(seqs, k_total, gather, backend, rank)
        for q in range(n_seq):
            ctx.compact(views[q], dviews[q], n_rows[q], seqs[q]["kept_idx"], seqs[q]["n_kept"], stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()

    clocks = ClockSampler(dev.index)
    with clocks:
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step()
            stream.synchronize()
            kept_total = sum(int(sq["n_kept"].sum()) for sq in seqs)
            barrier()
            torch.cuda.synchronize()
            l0 = ctx.launches()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                step()
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
            launches = ctx.launches() - l0
            ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.summary()
    if world > 1:
        t_ = torch.tensor([ms, kept_total], dtype=torch.float64, device=dev)
        m_ = t_.clone()
        dist.all_reduce(m_, op=dist.ReduceOp.MAX)
        dist.all_reduce(t_, op=dist.ReduceOp.SUM)
        ms, kept_total = float(m_[0]), int(t_[1])
    ctx.close()
    tria_b200.free(st)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    rows = int(n_kv.sum()) * c["L"] * KV
    step_b = rows * rb + 4 * kept_total * rb + 4 * rows + 8 * kept_total
    peak, peak_src = measured_peak()
    line = {
        "metric": METRIC, "value": rows / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32 (q8_0 cache)",
        "data": "synthetic (seeded device fill: N(0,1); seeded TRIA v2 stats; n_kv per sequence ~ U[8192, 16384])",
        "config": {"workload": f"{args.config}: {n_seq} sequences x {c['L']} layers x {KV} kv heads, "
                               f"n_kv {n_kv.tolist()}, head_dim {hd}, q8_0 K/V, global budget "
                               f"{c['budget']} rows per (layer, kv-head) per sequence",
                   "kept_rows": kept_total, "shard": f"contiguous layer blocks over {world} rank(s)",
                   "collectives": ("1 all-gather of per-sequence candidate scores per step" if one else
                                   "3 all-gathers of per-sequence key histograms / tie counts per step"),
                   "l2": "inputs larger than L2 (no flush)"},
        "step_roofline": {"bytes_per_step": step_b, "achieved": step_b / (ms / 1e3) / 1e9,
                          "frac": step_b / (ms / 1e3) / 1e9 / peak, "unit": "GB/s",
                          "peak_source": f"{peak_src} hbm_gbs"},
        "clocks": clk,
        "gpu_launches": int(launches),
        "e2e": None,
        "e2e_note": "device-resident batch; the host-buffer path is measured on the single-step configs",
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--no-graph", action="store_true",
                    help="time eager tria_evict calls instead of replaying the step captured in a CUDA graph")
    ap.add_argument("--global-protocol", default="histograms", choices=["histograms", "candidates"],
                    help="multiseq-q8_0-global: three all-gathers of key histograms, or one of candidates")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="N > 1: strong (default) = layers partitioned over the ranks; weak = a full cache per rank")
    ap.add_argument("--layers", type=int, default=0,
                    help="profile a smaller case: only the first N layers of the workload")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--ramp-sequence", action="store_true",
                    help="time the 5-step exponential ramp schedule (10/20/40/80/100%%, +128 rows between steps)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.scaling is None:
        args.scaling = "strong" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "weak"
    if args.layers:
        CONFIGS[args.config] = dict(CONFIGS[args.config], L=args.layers)
    if args.impl == "reference":
        run_reference(args)
    elif args.ramp_sequence:
        run_ramp(args)
    elif "seqs" in CONFIGS[args.config]:
        run_global(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
