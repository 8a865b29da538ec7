#!/usr/bin/env python
"""Benchmark of the fused residual-add + RMSNorm hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload sweep|config0|shard|decode|relu]

Prints ONE JSON line (rank 0).  Default workload ("sweep", BASELINE config 1,
the configuration the headline metric is quoted on): one step is one pass of
the fused op over batch 4096 bf16 at each of the 20 hidden sizes
1024..16384 (step 1024), 20480, 24576, 28672, 32768.  `value` is the
whole-job algorithmic HBM throughput in GB/s (bytes = 4*B*H*2 + 2*H per
launch: read input, residual, weight; write output, residual) with inputs
resident in HBM; `e2e` is the same metric through the C ABI with host
buffers, the host<->device copies inside the timed region.

Cold L2: every hidden size has its own buffers (4 GB per step in total, far
above the 126 MB L2), so each launch's data was last touched one full step
earlier; no flush is needed and nothing is cached between timed launches.

Multi-GPU (torchrun, one process per GPU): rows shard with no collective;
each rank runs the same per-GPU workload (weak scaling) and the step time is
the max over ranks.  `--workload shard` instead splits BASELINE config 4's
global batches (65536 x 8192 and 32768 x 32768) across the ranks (strong
scaling).

Every line also carries `strong`: BASELINE config 4's global batches split
over the ranks with shard.row_range, timed after the main region, next to the
same global problem on one GPU.

`--impl reference` times the reference's own CPU formula (the eager PyTorch
expression of its test, test/test_hp_rms_norm.py:6-19, restated in
oracle/oracle.py) on the host cores: one step is the full batch at one shape
of the workload (shape k mod 20 at step k), so 20 steps cover the sweep once.
Our arm's `cpu_baseline` runs the same code on one such pass.  Where a GPU and
the reference's CUDA kernels compiled here (oracle/_ref) are present, the
reference arm also times that kernel per shape on the GPU, the same way our
per-shape numbers are taken (`gpu_reference_kernel`).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SWEEP = [1024 * i for i in range(1, 17)] + [20480, 24576, 28672, 32768]
BATCH = 4096
ELEM = 2  # bytes per bf16 element
METRIC = "fused add+RMSNorm µs and achieved HBM GB/s (% of B200 peak), batch 4096 bf16"
# Reference README B200 table (CUDA 13.1 build, batch 4096 bf16), hp_rms_norm column, in us.
README_US = {1024: 9.34, 2048: 12.35, 3072: 15.23, 4096: 18.69, 5120: 23.78, 6144: 28.8,
             7168: 34.69, 8192: 39.9, 9216: 46.43, 10240: 51.42, 11264: 55.14, 12288: 59.78,
             13312: 80.38, 14336: 83.39, 15360: 86.4, 16384: 90.98, 20480: 115.74,
             24576: 137.31, 28672: 161.15, 32768: 182.34}
SHARD_SHAPES = [(65536, 8192), (32768, 32768)]
DECODE_ROWS = [1, 7, 33, 128, 512]
DECODE_HIDDEN = [4096, 5120, 7168, 8192]
RELU_SHAPES = [((4096, 14336), "bf16"), ((8192, 28672), "fp16")]


def alg_bytes(rows: int, hidden: int) -> int:
    return 4 * rows * hidden * ELEM + hidden * ELEM


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload",
                    choices=["sweep", "config0", "shard", "decode", "relu", "variants", "act"],
                    default="sweep")
    ap.add_argument("--hidden", default=None,
                    help="comma-separated hidden sizes: restrict the sweep (e.g. for ncu captures)")
    ap.add_argument("--rows", type=int, default=BATCH, help="batch rows of the sweep/config0")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU work budget of the cpu_baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-shape", action="store_true")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the config-4 split (strong scaling) measured after the main region")
    ap.add_argument("--out", default=None, help="also write the JSON line to this file")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    return args


# --------------------------------------------------------------------------
# Distributed plumbing (one process per GPU; no collective on the data path).

class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False

    def init(self, backend: str):
        import torch
        import torch.distributed as dist

        if self.world > 1 and not dist.is_initialized():
            kw = {"device_id": torch.device("cuda", self.local_rank)} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=180), **kw)
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist

            dist.barrier()

    def max(self, v: float, device=None) -> float:
        if not self.pg:
            return v
        import torch
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist

            dist.destroy_process_group()


# --------------------------------------------------------------------------
# Clock sampling during the timed region (NVML reads only).

class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.dev = device_index
        self.period = period_s
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = None
            try:
                import torch

                uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            except Exception:
                pass
            h = None
            if uuid:
                try:
                    h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
                except Exception:
                    h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            self._h = h
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as e:  # no NVML: report what we could not sample
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception as e:
                self.error = str(e)
                return
            time.sleep(self.period)

    def __exit__(self, *exc):
        self.stop()

    def stop(self):
        self._stop.set()
        if self._thread:
            self._thread.join()
            self._thread = None

    def mark(self) -> int:
        """Index of the next sample (bracket a region with two marks)."""
        return len(self.samples)

    def summary(self, region=None):
        """Median SM clock and every clock-event reason seen over the whole
        sampled span; with `region` = (start mark, end mark), also the samples
        taken inside it (the timed region)."""
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz,
               "reasons": [n for b, n in self.REASONS.items() if self.reasons & b and b != 0x1],
               "samples": len(self.samples), "period_ms": round(self.period * 1e3),
               "span": "warm-up, timed region, per-shape, strong-scaling and end-to-end phases",
               "source": "nvml"}
        if region is not None:
            inside = self.samples[region[0]:region[1]]
            out["timed_region_samples"] = len(inside)
            out["timed_region_sm_mhz"] = statistics.median(inside) if inside else None
        if self.error:
            out["error"] = self.error
        return out


# --------------------------------------------------------------------------
# Measurement helpers.

# Nominal B200 HBM3e bandwidth (~8 TB/s); fractions of it are reported next to
# the fraction of the measured copy bandwidth, which is the roofline denominator.
NOMINAL_HBM_GBS = 8000.0


def measured_peak():
    """Measured HBM copy bandwidth of this pool (driver-written), else fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return 6650.0, "fallback (6.65 TB/s)"


def committed_traffic():
    """Per-launch DRAM bytes from the committed ncu summary, keyed by hidden size."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return None


def make_rows(rows, hidden, dtype, device, seed):
    """BASELINE config-0 distributions, generated on the device from a seed."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(rows, hidden, generator=g, device=device, dtype=torch.float32).to(dtype)
    r = torch.randn(rows, hidden, generator=g, device=device, dtype=torch.float32).to(dtype)
    w = (1.0 + 0.1 * torch.randn(hidden, generator=g, device=device)).to(dtype)
    return x, w, r


def graph_launch_us(torch, fn, nsets, dev, reps=3):
    """Per-launch time of `fn(k, stream)` as a CUDA graph of back-to-back
    launches over `nsets` rotating buffer sets (one warm replay, then `reps`
    timed replays)."""
    L = max(16, nsets)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(0, s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for k in range(L):
            fn(k % nsets, s.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * L)


def per_shape_us(torch, launch, i, rows, h, dev, min_bytes=600e6, fi=None):
    """Cold per-launch time of shape i (and of FlashInfer's fused_add_rmsnorm
    on the same buffers, when `fi` is given): graphs of back-to-back launches
    over rotating buffer sets."""
    set_bytes = rows * h * ELEM * 2
    nsets = min(256, max(2, int(-(-min_bytes // set_bytes))))  # tiny shapes: <= 256 sets
    xs = [torch.randn(rows, h, device=dev).to(torch.bfloat16) for _ in range(nsets)]
    rs = [torch.randn(rows, h, device=dev).to(torch.bfloat16) for _ in range(nsets)]
    w = (1 + 0.1 * torch.randn(h, device=dev)).to(torch.bfloat16)
    us = graph_launch_us(torch, lambda k, sh: launch(i, sh, xs[k], rs[k]), nsets, dev)
    fi_us = None
    if fi is not None:
        def theirs(k, sh):
            with torch.cuda.stream(torch.cuda.ExternalStream(sh)):
                fi(xs[k], rs[k], w, eps=1e-6)
        try:
            fi_us = graph_launch_us(torch, theirs, nsets, dev)
        except Exception:
            fi_us = None
    del xs, rs
    torch.cuda.empty_cache()
    return us, fi_us


def host_threads() -> int:
    """All host threads this process may use (torchrun sets OMP_NUM_THREADS=1
    per rank; the CPU legs run on one rank only, so they take the lot)."""
    import torch

    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(n)
    return n


def cpu_reference(shapes, steps: int, warmup: int):
    """The reference's CPU formula on the host cores: both CPU legs (our
    arm's cpu_baseline and the reference arm) call this, so they time the same
    code on the same sample.  One step is the eager formula over the FULL
    batch of one shape of the workload (step k takes shape k mod len(shapes),
    so len(shapes) steps cover the whole workload once); inputs are generated
    on the host from seed 0 with BASELINE config 0's distributions.

    Returns (GB/s, seconds timed, threads, sample description)."""
    import torch

    from oracle import oracle as O

    threads = host_threads()
    cache = {}

    def data(i):
        if i not in cache:
            rows, hidden = shapes[i]
            g = torch.Generator().manual_seed(i)
            x = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
            r = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
            w = (1.0 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
            cache[i] = (x, w, r)
        return cache[i]

    n = len(shapes)
    for k in range(max(steps, warmup)):  # inputs made before any timing
        data(k % n)
    for k in range(warmup):
        x, w, r = data(k % n)
        O.eager_formula(x, r, w, 1e-6)
    total, t0 = 0, time.perf_counter()
    for k in range(steps):
        x, w, r = data(k % n)
        O.eager_formula(x, r, w, 1e-6)
        total += alg_bytes(*shapes[k % n])
    el = time.perf_counter() - t0
    desc = (f"reference eager formula (test/test_hp_rms_norm.py:6-19, restated in oracle/oracle.py) "
            f"on {threads} host threads; {steps} steps after {warmup} warm-up, one step = the full "
            f"batch at one of the {n} shapes in turn ({min(steps, n)} distinct shapes timed)")
    return total / el / 1e9, el, threads, desc


def workload_shapes(args, world: int, rank: int):
    """(shapes of one step on this rank, workload description, scaling)."""
    if args.workload == "sweep":
        hs = [int(h) for h in args.hidden.split(",")] if args.hidden else SWEEP
        shapes = [(args.rows, h) for h in hs]
        if hs == SWEEP and args.rows == BATCH:
            workload = ("config1: fused add+RMSNorm hidden sweep 1024..16384 step 1024 + 20480, "
                        "24576, 28672, 32768 at batch 4096 bf16 (20 launches per step)")
        else:
            workload = f"config1 subset: batch {args.rows} bf16, hidden {hs}"
        return shapes, workload, "weak"
    if args.workload == "config0":
        return [(args.rows, 4096)], f"config0: fused add+RMSNorm {args.rows} x 4096 bf16", "weak"
    if args.workload == "shard":
        from hp_rms_norm_b200.shard import row_range

        shapes = []
        for rows, h in SHARD_SHAPES:
            start, stop = row_range(rows, world, rank)
            shapes.append((stop - start, h))
        return shapes, ("config4: global 65536 x 8192 and 32768 x 32768 bf16, rows split evenly "
                        "across ranks, no collective"), "strong"
    shapes = [(r, h) for r in DECODE_ROWS for h in DECODE_HIDDEN]
    return shapes, "config2 shapes (bf16): rows {1,7,33,128,512} x hidden {4096,5120,7168,8192}", \
        "weak"


def line_config(args, shapes, workload, world):
    """The `config` object of the JSON line (both arms build it here)."""
    return {"workload": workload, "batch": BATCH if args.workload != "decode" else None,
            "shapes": [list(x) for x in shapes],
            "l2": "cold: separate buffers per shape, 4 GB touched per step >> 126 MB L2",
            "bytes_per_step": sum(alg_bytes(r, h) for r, h in shapes),
            "parallelism": f"rows sharded x{world}, no collective"}


# --------------------------------------------------------------------------
# Our implementation.

def run_ours(args, dist):
    import torch

    from hp_rms_norm_b200 import capi

    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    dist.init("nccl")
    capi.load()
    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream

    if args.workload == "variants":
        return run_variants(args, dist, dev, stream)
    if args.workload == "act":
        return run_act(args, dist, dev, stream)
    if args.workload == "relu":
        return run_relu(args, dist, dev, stream)

    # ---- problem list for one step --------------------------------------
    shapes, workload, scaling = workload_shapes(args, dist.world, dist.rank)
    clocks = ClockSampler(dev.index).__enter__()  # sampled over the whole GPU part of the run

    bufs = []
    for i, (rows, h) in enumerate(shapes):
        x, w, r = make_rows(rows, h, torch.bfloat16, dev, seed=1000 * dist.rank + i)
        bufs.append((x, w, r))
    plans = [capi.plan(rows, h, capi.DTYPE_BF16, x.data_ptr(), r.data_ptr())
             for (rows, h), (x, w, r) in zip(shapes, bufs)]
    step_bytes = sum(alg_bytes(rows, h) for rows, h in shapes)
    eps = 1e-6

    # Consecutive launches of the same kernel template form a group; the timed
    # loop records one event per group boundary (a handful per step), so the
    # dominant kernel's launch time is measured inside the timed region without
    # an event pair around every launch.
    kern_of = [p.split(":tpr")[0] for p in plans]
    groups = []  # (kernel, [shape indices])
    for i, k in enumerate(kern_of):
        if groups and groups[-1][0] == k:
            groups[-1][1].append(i)
        else:
            groups.append((k, [i]))

    def launch(i, stream_handle, x=None, r=None):
        rows, h = shapes[i]
        bx, bw, br = bufs[i]
        x = bx if x is None else x
        r = br if r is None else r
        capi.rms_norm(x.data_ptr(), bw.data_ptr(), r.data_ptr(), rows, h, h, h, eps,
                      capi.DTYPE_BF16, stream_handle)

    def one_step(evs=None):
        for g, (_, idx) in enumerate(groups):
            if evs is not None:
                evs[g].record(stream)
            for i in idx:
                launch(i, sh)
        if evs is not None:
            evs[len(groups)].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            one_step()
    torch.cuda.synchronize()
    dist.barrier()

    K = args.steps
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(len(groups) + 1)]
             for _ in range(K)]
    torch.cuda.synchronize()
    dist.barrier()
    region0 = clocks.mark()
    for k in range(K):
        one_step(marks[k])
    torch.cuda.synchronize()
    region1 = clocks.mark()
    dist.barrier()
    elapsed_ms = dist.max(marks[0][0].elapsed_time(marks[K - 1][len(groups)]), dev)
    ms_per_step = elapsed_ms / K
    total_bytes = dist.world * step_bytes if scaling == "weak" else \
        sum(alg_bytes(r, h) for r, h in SHARD_SHAPES)
    value = total_bytes * K / (elapsed_ms / 1e3) / 1e9

    # ---- roofline of the dominant kernel (from the timed region) -----------
    peak, peak_src = measured_peak()
    by_kern = {}
    for g, (kern, idx) in enumerate(groups):
        t = sum(marks[k][g].elapsed_time(marks[k][g + 1]) for k in range(K)) / K * 1e3
        b = sum(alg_bytes(*shapes[i]) for i in idx)
        t0, b0, n0 = by_kern.get(kern, (0.0, 0, 0))
        by_kern[kern] = (t0 + t, b0 + b, n0 + len(idx))
    dom = max(by_kern, key=lambda k: by_kern[k][0])
    t_us, b_dom, n_dom = by_kern[dom]
    achieved = b_dom / t_us / 1e3
    traffic = None
    tr = committed_traffic()
    if tr:
        vals = [tr.get(str(shapes[i][1])) for i, k in enumerate(kern_of) if k == dom]
        if vals and all(v is not None for v in vals):
            traffic = int(sum(vals) / len(vals))
    roofline = {"bound": "hbm", "kernel": dom, "launches_per_step": n_dom,
                "time_share": round(t_us / sum(v[0] for v in by_kern.values()), 3),
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 3), "peak_source": peak_src,
                "avg_launch_us": round(t_us / n_dom, 2),
                "algorithmic_bytes_per_launch": int(b_dom / n_dom), "traffic": traffic,
                "traffic_source": ("from committed profile: profiles/traffic.json (ncu "
                                   "dram__bytes_read.sum + dram__bytes_write.sum of the same "
                                   "kernel and shapes, one launch each), not measured in this run")
                if traffic is not None else None}

    # ---- per-shape breakdown (after the timed region) ----------------------
    # Each shape alone: a CUDA graph of back-to-back launches over enough
    # rotating buffer sets (>= 600 MB) that every launch reads cold data;
    # FlashInfer's fused_add_rmsnorm (a library comparator) timed the same way.
    per_shape, plan_groups = [], {}
    fi = flashinfer_fused_add_rmsnorm() if not args.no_per_shape else None
    if not args.no_per_shape:
        for i, (rows, h) in enumerate(shapes):
            us, fi_us = per_shape_us(torch, launch, i, rows, h, dev, fi=fi)
            b = alg_bytes(rows, h)
            entry = [h, round(us, 2), round(b / us / 1e3 / peak, 3),
                     round(fi_us, 2) if fi_us is not None else None]
            if rows != BATCH:
                entry.append(rows)
            per_shape.append(entry)
            plan_groups.setdefault(plans[i], []).append(h)

    # ---- config 4 split over the ranks (strong scaling), every line ---------
    strong = None
    if not args.no_strong:
        strong = run_strong(dist, dev, peak)

    line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": dist.world,
            "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded on device: input, residual ~ N(0,1), weight ~ N(1,0.1), "
                    "eps 1e-6)",
            "config": line_config(args, shapes, workload, dist.world),
            "frac_of_peak": round(value / dist.world / peak, 3),
            "frac_of_nominal_peak": round(value / dist.world / NOMINAL_HBM_GBS, 3),
            "gpu_launches": K * len(shapes),
            "gpu_launches_note": "one hprn_rms_norm kernel launch per shape per timed step",
            "roofline": roofline}
    if args.workload == "sweep" and shapes == [(BATCH, h) for h in SWEEP]:
        readme_gbs = sum(alg_bytes(BATCH, h) for h in SWEEP) / (sum(README_US.values()) * 1e3)
        line["vs_baseline"] = round(value / dist.world / readme_gbs, 3)
        line["baseline_note"] = ("vs_baseline = per-GPU value / the reference README's B200 "
                                 f"aggregate over the same 20 shapes ({readme_gbs:.1f} GB/s, "
                                 "README.md:13-32, CUDA 13.1, L2 state unstated)")

    # ---- end to end through the C ABI with host buffers --------------------
    if not args.no_e2e and args.workload in ("sweep", "config0", "shard"):
        line["e2e"] = run_e2e(args, shapes, bufs, stream, dev, dist, eps)
    clocks.stop()
    line["clocks"] = clocks.summary((region0, region1))
    del bufs
    torch.cuda.empty_cache()

    # ---- CPU baseline (rank 0, N = 1): one pass of the workload ------------
    if dist.world == 1 and not args.no_cpu_baseline:
        gbs, _, threads, desc = cpu_reference(shapes, len(shapes), args.warmup)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                                "kind": "port", "sample": desc}
    if strong is not None:
        line["strong"] = strong
    if per_shape:
        # Last in the line, so the driver's stdout tail keeps every shape.
        line["plans"] = plan_groups
        line["per_shape_fields"] = ["hidden", "us", "frac_of_peak", "flashinfer_us"] + \
            (["rows"] if any(len(e) > 4 for e in per_shape) else [])
        line["per_shape_method"] = ("each shape alone, CUDA-graph replay of back-to-back launches "
                                    "over rotating buffer sets (>= 600 MB), cold L2; FlashInfer "
                                    "fused_add_rmsnorm timed the same way")
        line["per_shape"] = per_shape
    return line


def flashinfer_fused_add_rmsnorm():
    """FlashInfer's fused_add_rmsnorm(input, residual, weight, eps) where it is
    installed (a library comparator: timed next to ours, never used by ours)."""
    try:
        from flashinfer.norm import fused_add_rmsnorm
    except Exception:
        return None
    return fused_add_rmsnorm


def run_strong(dist, dev, peak, steps: int = 10, warmup: int = 3):
    """BASELINE config 4 at this world size: each global batch (65536 x 8192
    and 32768 x 32768 bf16) split over the ranks with shard.row_range, each
    rank running its rows on its own GPU (no collective); one step = both
    shapes.  Next to it, the same global problem on one GPU (each rank's own
    GPU; the fastest counts), which is the 1-GPU figure the efficiency divides
    by.  Times are CUDA events over `steps` steps, max over ranks."""
    import torch

    from hp_rms_norm_b200 import capi
    from hp_rms_norm_b200.shard import row_range

    stream = torch.cuda.Stream(device=dev)

    def step_ms(parts):
        def step():
            for rows, h, (x, w, r) in parts:
                capi.rms_norm(x.data_ptr(), w.data_ptr(), r.data_ptr(), rows, h, h, h, 1e-6,
                              capi.DTYPE_BF16, stream.cuda_stream)

        with torch.cuda.stream(stream):
            for _ in range(warmup):
                step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        return e0.elapsed_time(e1) / steps

    def alloc(rows_of):
        return [(rows_of(R), h, make_rows(rows_of(R), h, torch.bfloat16, dev, seed=77 + i))
                for i, (R, h) in enumerate(SHARD_SHAPES)]

    share = alloc(lambda R: row_range(R, dist.world, dist.rank)[1] - row_range(R, dist.world,
                                                                               dist.rank)[0])
    t_share = step_ms(share)
    rows_here = [p[0] for p in share]
    del share
    torch.cuda.empty_cache()
    if dist.world > 1:
        full = alloc(lambda R: R)
        t_full = step_ms(full)
        del full
        torch.cuda.empty_cache()
    else:
        t_full = t_share
    t_slow = dist.max(t_share, dev)
    t_one = -dist.max(-t_full, dev)  # the fastest GPU's time for the global problem
    total = sum(alg_bytes(R, h) for R, h in SHARD_SHAPES)
    agg = total / (t_slow / 1e3) / 1e9
    one = total / (t_one / 1e3) / 1e9
    return {"workload": "config4: global 65536 x 8192 + 32768 x 32768 bf16 per step, rows split "
                        "with shard.row_range, no collective",
            "rows_per_rank": rows_here, "steps": steps,
            "aggregate_gbs": round(agg, 1), "per_gpu_frac": round(agg / dist.world / peak, 3),
            "one_gpu_gbs": round(one, 1), "efficiency": round(agg / (dist.world * one), 3),
            "slowest_rank_us": round(t_slow * 1e3, 1), "one_gpu_us": round(t_one * 1e3, 1),
            "limiter": ("per-rank launch size: each rank runs 1/N of the rows as one launch per "
                        "shape; no collective and no data crosses NVLink")}


def run_e2e(args, shapes, bufs, stream, dev, dist, eps):
    """Same metric through the C ABI with pinned host buffers: per step, every
    shape's input, residual and weight go host->device, the kernel runs, and the
    output and residual come back device->host.  Chunks of rows rotate over
    three streams so the two copy directions overlap."""
    import torch

    from hp_rms_norm_b200 import capi

    host = []
    for (rows, h), (x, w, r) in zip(shapes, bufs):
        host.append((x.cpu().pin_memory(), w.cpu().pin_memory(), r.cpu().pin_memory(),
                     torch.empty_like(x, device="cpu").pin_memory(),
                     torch.empty_like(r, device="cpu").pin_memory()))
    streams = [torch.cuda.Stream(device=dev) for _ in range(3)]
    chunk_bytes = 64 << 20  # input + residual bytes per chunk
    h2d = sum(x.numel() * 2 + r.numel() * 2 + w.numel() * 2 for x, w, r in bufs)
    d2h = sum(x.numel() * 2 + r.numel() * 2 for x, w, r in bufs)

    def step():
        main = torch.cuda.current_stream()
        for (_, w, _), (_, hw, _, _, _) in zip(bufs, host):
            w.copy_(hw, non_blocking=True)
        for s in streams:
            s.wait_stream(main)
        # Every shape's row chunks rotate over the streams without a join in
        # between, so host->device copies of one chunk overlap device->host
        # copies of another across shape boundaries too.
        c = 0
        for (rows, h), (x, w, r), (hx, hw, hr, ox, orr) in zip(shapes, bufs, host):
            per = max(1, chunk_bytes // (h * 2 * 2))
            for r0 in range(0, rows, per):
                r1 = min(rows, r0 + per)
                s = streams[c % len(streams)]
                c += 1
                with torch.cuda.stream(s):
                    x[r0:r1].copy_(hx[r0:r1], non_blocking=True)
                    r[r0:r1].copy_(hr[r0:r1], non_blocking=True)
                    capi.rms_norm(x[r0:r1].data_ptr(), w.data_ptr(), r[r0:r1].data_ptr(), r1 - r0,
                                  h, h, h, eps, capi.DTYPE_BF16, s.cuda_stream)
                    ox[r0:r1].copy_(x[r0:r1], non_blocking=True)
                    orr[r0:r1].copy_(r[r0:r1], non_blocking=True)
        for s in streams:
            main.wait_stream(s)

    for _ in range(1):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    K = max(1, args.e2e_steps)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(K):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = dist.max(t0.elapsed_time(t1), dev) / K
    total = sum(alg_bytes(rows, h) for rows, h in shapes) * dist.world
    value = total / (ms / 1e3) / 1e9
    link = pcie_ceiling(dev)
    return {"value": round(value, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3),
            "steps": K, "api": "hprn_rms_norm (C ABI) on pinned-host-staged buffers, 3 streams",
            "roofline": {"bound": "pcie", "achieved": round(value / dist.world, 2),
                         "peak": link["bidirectional_gbs"], "unit": "GB/s",
                         "frac": round(value / dist.world / link["bidirectional_gbs"], 3),
                         "peak_source": "measured here: " + link["how"], **link}}


def pcie_ceiling(dev, nbytes=1 << 30, reps=3):
    """Host<->device copy bandwidth of this GPU's link, measured live: pinned
    buffers of `nbytes`, H2D alone, D2H alone, and both at once on two streams
    (the bound of the end-to-end number, whose steps move as many bytes each
    way)."""
    import torch

    n = nbytes // 2
    h_in = torch.empty(n, dtype=torch.bfloat16).pin_memory()
    h_out = torch.empty(n, dtype=torch.bfloat16).pin_memory()
    d_a = torch.empty(n, dtype=torch.bfloat16, device=dev)
    d_b = torch.empty(n, dtype=torch.bfloat16, device=dev)
    s1, s2 = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps / 1e3

    def both():
        main = torch.cuda.current_stream()
        s1.wait_stream(main)
        s2.wait_stream(main)
        with torch.cuda.stream(s1):
            d_a.copy_(h_in, non_blocking=True)
        with torch.cuda.stream(s2):
            h_out.copy_(d_b, non_blocking=True)
        main.wait_stream(s1)
        main.wait_stream(s2)

    h2d = nbytes / timed(lambda: d_a.copy_(h_in, non_blocking=True)) / 1e9
    d2h = nbytes / timed(lambda: h_out.copy_(d_b, non_blocking=True)) / 1e9
    bi = 2 * nbytes / timed(both) / 1e9
    return {"h2d_gbs": round(h2d, 1), "d2h_gbs": round(d2h, 1), "bidirectional_gbs": round(bi, 1),
            "how": f"pinned {nbytes >> 20} MiB copies, both directions at once on two streams"}


VARIANT_HIDDEN = [2048, 4096, 8192, 16384, 32768]
# name -> (residual?, output form, algorithmic bytes per element)
VARIANTS = {
    "fused_in_place": (True, "same", 8),
    "fused_out_of_place": (True, "same", 8),
    "plain": (False, "same", 4),
    "fused_fp8_static": (True, "fp8s", 7),
    "fused_fp8_dynamic": (True, "fp8d", 7),
    "plain_fp8_dynamic": (False, "fp8d", 3),
    "fused_nvfp4": (True, "nvfp4", 6.5625),   # + e2m1 codes 0.5 B and a scale byte per 16
    "plain_nvfp4": (False, "nvfp4", 2.5625),
    "fused_fp8_group128": (True, "fp8g", 7.03125),  # + one float32 scale per 128 elements
    "plain_fp8_group128": (False, "fp8g", 3.03125),
}


# Graph replays per shape in the variants workload (each replay is >= 16
# launches over rotating cold buffer sets).
VARIANT_WARMUP = 3
VARIANT_STEPS = 3


def run_variants(args, dist, dev, stream):
    """Extended forms (plain RMSNorm, out-of-place, fp8 outputs) at batch 4096
    bf16 and hidden 2048..32768: per-variant GB/s over its algorithmic bytes
    (inputs read once, outputs written once; fp8 output 1 byte per element,
    plus 4 bytes per row of scales for the dynamic form), each shape timed as
    graph replays over rotating cold buffers."""
    import torch

    from hp_rms_norm_b200 import capi

    rows = args.rows
    peak, peak_src = measured_peak()
    results = {}
    for name, (res, form, bpe) in VARIANTS.items():
        per = []
        for h in ([int(x) for x in args.hidden.split(",")] if args.hidden else VARIANT_HIDDEN):
            set_bytes = rows * h * 2 * 2
            nsets = max(2, int(-(-600e6 // set_bytes)))
            xs = [torch.randn(rows, h, device=dev).to(torch.bfloat16) for _ in range(nsets)]
            rs = [torch.randn(rows, h, device=dev).to(torch.bfloat16) for _ in range(nsets)]
            w = (1 + 0.1 * torch.randn(h, device=dev)).to(torch.bfloat16)
            if form == "same":
                outs = xs if name == "fused_in_place" else \
                    [torch.empty(rows, h, device=dev, dtype=torch.bfloat16) for _ in range(nsets)]
            elif form == "nvfp4":
                outs = [torch.empty(rows, h // 2, device=dev, dtype=torch.uint8)
                        for _ in range(nsets)]
            else:
                outs = [torch.empty(rows, h, device=dev, dtype=torch.float8_e4m3fn)
                        for _ in range(nsets)]
            scale = torch.tensor([0.01 if form != "nvfp4" else 336.0], device=dev)
            rsc = torch.empty(rows, device=dev)
            gsc = torch.empty(rows, h // 128, device=dev)
            bsc = torch.empty(rows, h // 16, device=dev, dtype=torch.uint8)

            def call(k, sh, h=h, xs=xs, rs=rs, w=w, outs=outs, form=form, res=res):
                if form == "fp8g":
                    capi.rms_norm_fp8_group(outs[k].data_ptr(), gsc.data_ptr(), h // 128, 1,
                                            xs[k].data_ptr(), w.data_ptr(),
                                            rs[k].data_ptr() if res else None, rows, h, h, h, h,
                                            1e-6, capi.DTYPE_BF16, 128, False, sh)
                    return
                if form == "nvfp4":
                    capi.rms_norm_nvfp4(outs[k].data_ptr(), bsc.data_ptr(), xs[k].data_ptr(),
                                        w.data_ptr(), rs[k].data_ptr() if res else None, rows, h,
                                        h, h, h, 1e-6, capi.DTYPE_BF16, scale.data_ptr(), sh)
                    return
                ocode = {"same": capi.OUT_SAME, "fp8s": capi.OUT_FP8_E4M3_STATIC,
                         "fp8d": capi.OUT_FP8_E4M3_DYNAMIC}[form]
                capi.rms_norm_out(outs[k].data_ptr(), xs[k].data_ptr(), w.data_ptr(),
                                  rs[k].data_ptr() if res else None, rows, h, h, h, h, 1e-6,
                                  capi.DTYPE_BF16, ocode, scale.data_ptr(), rsc.data_ptr(), sh)

            L = max(16, nsets)
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                call(0, s.cuda_stream)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for k in range(L):
                    call(k % nsets, s.cuda_stream)
            for _ in range(VARIANT_WARMUP):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(VARIANT_STEPS):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (VARIANT_STEPS * L)
            byt = int(rows * h * bpe) + h * 2 + (rows * 4 if form == "fp8d" else 0)
            per.append({"hidden": h, "us": round(us, 2), "gbs": round(byt / us / 1e3, 1),
                        "frac": round(byt / us / 1e3 / peak, 3)})
            del g, xs, rs, outs
            torch.cuda.empty_cache()
        tot_b = sum(e["gbs"] * e["us"] for e in per)
        tot_t = sum(e["us"] for e in per)
        results[name] = {"gbs": round(tot_b / tot_t, 1), "frac": round(tot_b / tot_t / peak, 3),
                         "per_shape": per}
    value = statistics.mean(v["gbs"] for v in results.values())
    return {"metric": "extended RMSNorm forms: achieved HBM GB/s (bf16 input, batch 4096)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": dist.world,
            "steps": VARIANT_STEPS, "warmup": VARIANT_WARMUP, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic N(0,1)",
            "config": {"workload": "variants", "rows": rows,
                       "hidden": [e["hidden"] for e in next(iter(results.values()))["per_shape"]],
                       "bytes_per_element": {k: v[2] for k, v in VARIANTS.items()},
                       "l2": "cold: rotating buffer sets >= 600 MB, graph replays"},
            "peak": peak, "peak_source": peak_src, "variants": results}


def run_act(args, dist, dev, stream):
    """Gated activations (silu/gelu/gelu_tanh-and-mul) on a [4096, 2 x 14336]
    bf16 input (an LLM MLP's gate/up projection): GB/s over 6 bytes per output
    element (gate and up read, out written)."""
    import torch

    from hp_rms_norm_b200 import capi

    rows, d = args.rows, 14336
    peak, peak_src = measured_peak()
    nsets = 3
    xs = [torch.randn(rows, 2 * d, device=dev).to(torch.bfloat16) for _ in range(nsets)]
    outs = [torch.empty(rows, d, device=dev, dtype=torch.bfloat16) for _ in range(nsets)]
    results = {}
    for name, act in (("silu", capi.ACT_SILU), ("gelu", capi.ACT_GELU),
                      ("gelu_tanh", capi.ACT_GELU_TANH)):
        def step(k, sh, act=act):
            capi.act_and_mul(outs[k].data_ptr(), xs[k].data_ptr(), rows, d, d, 2 * d, act,
                             capi.DTYPE_BF16, sh)

        with torch.cuda.stream(stream):
            for k in range(args.warmup):
                step(k % nsets, stream.cuda_stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(args.steps):
            step(k % nsets, stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        byt = rows * d * 6
        results[name] = {"us": round(us, 2), "gbs": round(byt / us / 1e3, 1),
                         "frac": round(byt / us / 1e3 / peak, 3)}
    value = statistics.mean(v["gbs"] for v in results.values())
    return {"metric": "gated activation (act(gate) * up) achieved HBM GB/s", "value": round(value, 1),
            "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1)",
            "config": {"workload": f"act_and_mul [{rows}, 2x{d}] bf16",
                       "l2": "3 rotating input/output sets of 352 MB"},
            "peak": peak, "peak_source": peak_src, "activations": results}


def run_relu(args, dist, dev, stream):
    import torch

    from hp_rms_norm_b200 import capi

    bufs = []
    for (shape, dt) in RELU_SHAPES:
        tdt = torch.bfloat16 if dt == "bf16" else torch.float16
        g = torch.Generator(device=dev).manual_seed(3 + dist.rank)
        x = torch.randn(shape, generator=g, device=dev).to(tdt)
        bufs.append((x, torch.empty_like(x), capi.DTYPE_BF16 if dt == "bf16" else capi.DTYPE_FP16))
    step_bytes = sum(2 * x.numel() * 2 for x, _, _ in bufs)

    def one_step():
        for x, o, code in bufs:
            capi.relu(o.data_ptr(), x.data_ptr(), x.shape[0], x.shape[1], x.shape[1], x.shape[1],
                      code, stream.cuda_stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            one_step()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            one_step()
        end.record(stream)
        torch.cuda.synchronize()
    ms = dist.max(start.elapsed_time(end), dev) / args.steps
    peak, src = measured_peak()
    value = dist.world * step_bytes / (ms / 1e3) / 1e9
    return {"metric": "elementwise ReLU achieved HBM GB/s", "value": round(value, 1),
            "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16+fp16", "data": "synthetic N(0,1)",
            "config": {"workload": "config3: relu bf16 (4096,14336) + fp16 (8192,28672)",
                       "l2": "inputs 112 MiB + 448 MiB per step"},
            "roofline": {"bound": "hbm", "achieved": round(value / dist.world, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(value / dist.world / peak, 3),
                         "peak_source": src, "traffic": None},
            "gpu_launches": args.steps * len(bufs), "clocks": clocks.summary()}


# --------------------------------------------------------------------------
# The reference arm: the reference's CPU formula on the host cores.

def run_reference(args, dist):
    import torch

    if dist.rank != 0:
        return None
    shapes, workload, _ = workload_shapes(args, 1, 0)
    gbs, el, threads, desc = cpu_reference(shapes, args.steps, args.warmup)
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded on the host: input, residual ~ N(0,1), weight ~ N(1,0.1), "
                    "eps 1e-6)",
            "config": line_config(args, shapes, workload, 1),
            "impl": "reference",
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                             "kind": "port", "sample": desc},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if torch.cuda.is_available() and not args.no_per_shape and args.workload == "sweep":
        line["gpu_reference_kernel"] = reference_kernel_per_shape(shapes)
    return line


def reference_kernel_per_shape(shapes):
    """The reference's own CUDA kernel (launch_rms_norm, compiled from the
    reference sources into oracle/_ref by oracle/build.py) timed per shape on
    GPU 0 exactly as our arm times its per-shape numbers: a CUDA graph of
    back-to-back launches over rotating buffer sets of >= 600 MB (cold L2).
    A same-box comparator, reported beside the CPU value; "error" where the
    reference rejects the shape (its CUDA-12 build: hidden >= 24576)."""
    import torch

    from oracle import oracle as O

    try:
        ref = O.ReferenceKernels()
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {e}"}
    dev = torch.device("cuda", 0)
    out = []
    for rows, h in shapes:
        nsets = min(256, max(2, int(-(-600e6 // (rows * h * ELEM * 2)))))
        xs = [torch.randn(rows, h, device=dev).to(torch.bfloat16) for _ in range(nsets)]
        rs = [torch.randn(rows, h, device=dev).to(torch.bfloat16) for _ in range(nsets)]
        w = (1 + 0.1 * torch.randn(h, device=dev)).to(torch.bfloat16)
        try:
            us = graph_launch_us(torch, lambda k, sh: ref.rms_norm(xs[k], w, rs[k], 1e-6, sh),
                                 nsets, dev)
            out.append([h, round(us, 2)])
        except RuntimeError as e:
            out.append([h, "error: " + str(e).splitlines()[0][:40]])
        del xs, rs
        torch.cuda.empty_cache()
    return {"fields": ["hidden", "us"], "rows": shapes[0][0],
            "method": "CUDA-graph replay of back-to-back launches over rotating buffer sets "
                      "(>= 600 MB), cold L2, as our per_shape",
            "source": "reference launch_rms_norm compiled here from its sources (CUDA 12.9, sm_100a)",
            "per_shape": out}


def main():
    args = parse_args()
    dist = Dist()
    if args.impl == "reference":
        line = run_reference(args, dist)
    else:
        line = run_ours(args, dist)
    if line is not None and dist.rank == 0:
        s = json.dumps(line)
        print(s, flush=True)
        if args.out:
            with open(args.out, "w") as f:
                f.write(s + "\n")
    dist.close()


if __name__ == "__main__":
    main()
