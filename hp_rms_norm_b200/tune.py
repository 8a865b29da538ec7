"""Launch-plan sweep for the fused add + RMSNorm kernels.

    python -m hp_rms_norm_b200.tune [--rows 4096] [--hidden 1024,2048,...]
                                    [--dtype bf16|fp16] [--warm] [--json out.json]
                                    [--no-tma | --tma-only] [--isolated] [--copy]
                                    [--default-only] [--knobs]
                                    [--variant fused|fused_out|plain|fused_fp8s|fused_fp8d|
                                               plain_fp8s|plain_fp8d|fused_nvfp4|plain_nvfp4|
                                               fused_fp8g|plain_fp8g]

Times every compiled launch plan that covers each requested shape (through
``hprn_set_plan_override``) and prints the fastest, next to the built-in
heuristic's choice.  Candidates: warp rows (one warp per row, or several
short rows per warp), one CTA per row and clusters of 2/4/8 CTAs at 32-byte
vectors, one CTA per row at 16-byte vectors, two passes (one CTA or a
cluster per row) past 4096 vectors, and TMA-staged rows (unless
``--no-tma``).  ``--copy`` also times torch's ``copy_`` of the same bytes.  ``--knobs``
times the default plan under each pair of launch knobs instead
(``default:pf<p>:et<e>``: L2 prefetch before the programmatic-launch wait in
no CTA, the first wave or every CTA, or the first wave with every CTA also
prefetching the row one wave ahead; dependents triggered after the last store,
after the row reduction, or once the loads are issued), one process per pair,
which is how
``default_knobs`` in csrc/rms_norm.cu was fitted.  Timing: a CUDA graph of
back-to-back launches over
rotating buffer sets of at least 600 MB, so every launch reads cold data (or
one buffer set with ``--warm``), replayed three times after one warm replay;
with ``--isolated``, the median of single launches each preceded by an L2
flush.

This is how the heuristic in csrc/rms_norm.cu (``default_plan``) was fitted on
B200; rerun it to check the heuristic on another part or other shapes.
"""
from __future__ import annotations

import argparse
import json
import math

SWEEP = [1024 * i for i in range(1, 17)] + [20480, 24576, 28672, 32768]


# variant: (adds a residual, output form, algorithmic bytes per element)
VARIANTS = {
    "fused": (True, "same", 8),        # the reference's in-place form
    "fused_out": (True, "same", 8),
    "plain": (False, "same", 4),
    "fused_fp8s": (True, "fp8s", 7),
    "fused_fp8d": (True, "fp8d", 7),
    "plain_fp8s": (False, "fp8s", 3),
    "plain_fp8d": (False, "fp8d", 3),
    "fused_nvfp4": (True, "nvfp4", 6.5625),
    "plain_nvfp4": (False, "nvfp4", 2.5625),
    "fused_fp8g": (True, "fp8g", 7.03125),   # group-128 scales
    "plain_fp8g": (False, "fp8g", 3.03125),
}


# Shared memory one CTA may use for a TMA ring on B200 (227 KB, less the
# kernel's mbarriers and partials).
TMA_SMEM = 232448 - 1024


def tma_candidates(hidden: int, residual: bool) -> list[str]:
    """TMA-staged plans (16- or 32-byte vectors, persistent grid) covering
    `hidden`, for ring depths whose buffers fit one CTA."""
    stage = (2 if residual else 1) * hidden * 2
    out = []
    for vec in (16, 32):
        if hidden % (vec // 2):
            continue
        nv = hidden // (vec // 2)
        for vpt in (1, 2, 4, 8):
            load = vpt * vec // 16  # 16-byte pieces per thread
            max_threads = 1024 if load <= 2 else (512 if load <= 4 else 256)
            tpr = -(-(-(-nv // vpt)) // 32) * 32
            if tpr > max_threads or (tpr > 32 and (tpr - 32) * vpt >= nv):
                continue
            out += [f"tma:vec{vec}:vpt{vpt}:tpr{tpr}:cluster1:rpc{st}"
                    for st in (1, 2, 3, 4, 6, 8) if st * stage <= TMA_SMEM]
    return out


def candidates(nvec: int, full: bool = True) -> list[str]:
    """Plans (32-byte vectors) whose threads x vectors x CTAs cover nvec vectors
    (full: the in-place fused form's plan set; else the extended forms' set)."""
    out = []
    warp_vpts = (1, 2, 3, 4) if full else (1, 2, 4)
    cta_vpts = (1, 2, 3, 4, 6, 8) if full else (1, 2, 4)
    if nvec <= 128:
        vpt = min(v for v in warp_vpts if v * 32 >= nvec)
        out += [f"warp:vec32:vpt{vpt}:tpr32:cluster1:rpc{r}" for r in (2, 4, 8)]
    if nvec <= 64:  # several short rows per warp: tpr lanes per row
        for lanes in (1, 2, 4, 8, 16):
            vpt = -(-nvec // lanes)
            if vpt in warp_vpts:
                out += [f"warp:vec32:vpt{vpt}:tpr{lanes}:cluster1:rpc{t // lanes}" for t in (128, 256)]
    for cl in (1, 2, 4, 8):
        for vpt in cta_vpts:
            max_threads = 1024 if vpt <= 2 else (512 if vpt <= 4 else 256)
            sl = -(-nvec // cl)
            tpr = -(-(-(-sl // vpt)) // 32) * 32
            if tpr > max_threads or (tpr > 32 and (tpr - 32) * vpt >= sl):
                continue
            kind = "cta" if cl == 1 else "cluster"
            out.append(f"{kind}:vec32:vpt{vpt}:tpr{tpr}:cluster{cl}:rpc1")
    # 16-byte vectors (twice the threads for the same row) for rows that fit
    # one CTA: more, smaller accesses in flight per row.
    n16 = 2 * nvec
    for vpt in (1, 2):
        tpr = -(-(-(-n16 // vpt)) // 32) * 32
        if 32 <= tpr <= 1024:
            out.append(f"cta:vec16:vpt{vpt}:tpr{tpr}:cluster1:rpc1")
    if n16 <= 128:
        vpt16 = -(-n16 // 32)
        if vpt16 in warp_vpts:
            out += [f"warp:vec16:vpt{vpt16}:tpr32:cluster1:rpc{r}" for r in (4, 8)]
    if nvec > 4096:  # two passes, one CTA or a cluster per row
        out += [f"twopass:vec32:vpt4:tpr{t}:cluster{cl}:rpc1" for cl in (1, 2, 4, 8)
                for t in (128, 256, 512)]
    return out


def graph_us(torch, fn, nsets: int, reps: int = 3) -> float:
    L = max(24, nsets)
    s = torch.cuda.Stream()
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
    return e0.elapsed_time(e1) * 1e3 / (reps * L)


def isolated_us(torch, fn, nsets: int, flush, reps: int = 7) -> float:
    """Median time of one launch on its own: L2 flushed (a write of a buffer
    larger than L2), then the launch alone between two events."""
    s = torch.cuda.current_stream()
    ts = []
    for k in range(reps + 1):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn(k % nsets, s.cuda_stream)
        e1.record()
        torch.cuda.synchronize()
        if k:
            ts.append(e0.elapsed_time(e1) * 1e3)
    return sorted(ts)[len(ts) // 2]


def sweep(rows: int, hiddens: list[int], dtype: str = "bf16", warm: bool = False,
          variant: str = "fused", tma: bool = True, tma_only: bool = False,
          isolated: bool = False, copy: bool = False, default_only: bool = False) -> dict:
    import torch

    from . import capi

    res_needed, form_name, bpe = VARIANTS[variant]
    form = {"same": capi.OUT_SAME, "fp8s": capi.OUT_FP8_E4M3_STATIC,
            "fp8d": capi.OUT_FP8_E4M3_DYNAMIC, "nvfp4": capi.OUT_NVFP4,
            "fp8g": capi.OUT_FP8_E4M3_GROUP}[form_name]

    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    code = capi.DTYPE_BF16 if dtype == "bf16" else capi.DTYPE_FP16
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if isolated else None
    time_us = (lambda fn, n: isolated_us(torch, fn, n, flush)) if isolated else \
        (lambda fn, n: graph_us(torch, fn, n))
    results = {}
    for h in hiddens:
        set_bytes = rows * h * 2 * 2
        nsets = 1 if warm else max(3, min(512, math.ceil(600e6 / set_bytes)))
        xs = [torch.randn(rows, h, device=dev).to(tdt) for _ in range(nsets)]
        rs = [torch.randn(rows, h, device=dev).to(tdt) for _ in range(nsets)]
        w = (1 + 0.1 * torch.randn(h, device=dev)).to(tdt)
        fp8 = form != capi.OUT_SAME
        if variant == "fused":
            outs = xs
        elif form == capi.OUT_NVFP4:
            outs = [torch.empty(rows, h // 2, device=dev, dtype=torch.uint8) for _ in range(nsets)]
        else:
            outs = [torch.empty(rows, h, device=dev,
                                dtype=torch.float8_e4m3fn if fp8 else tdt) for _ in range(nsets)]
        scale = torch.tensor([0.01 if form != capi.OUT_NVFP4 else 336.0], device=dev)
        row_scales = torch.empty(rows, device=dev)
        block_scales = torch.empty(rows, max(1, h // 16), device=dev, dtype=torch.uint8)
        byt = int(rows * h * bpe) + 2 * h + (4 * rows if form_name == "fp8d" else 0)

        group_scales = torch.empty(rows, max(1, h // 128), device=dev)

        def run(k, s):
            if form == capi.OUT_FP8_E4M3_GROUP:
                capi.rms_norm_fp8_group(outs[k].data_ptr(), group_scales.data_ptr(), h // 128, 1,
                                        xs[k].data_ptr(), w.data_ptr(),
                                        rs[k].data_ptr() if res_needed else None, rows, h, h, h, h,
                                        1e-6, code, 128, False, s)
                return
            if form == capi.OUT_NVFP4:
                capi.rms_norm_nvfp4(outs[k].data_ptr(), block_scales.data_ptr(), xs[k].data_ptr(),
                                    w.data_ptr(), rs[k].data_ptr() if res_needed else None, rows,
                                    h, h, h, h, 1e-6, code, scale.data_ptr(), s)
                return
            capi.rms_norm_out(outs[k].data_ptr(), xs[k].data_ptr(), w.data_ptr(),
                              rs[k].data_ptr() if res_needed else None, rows, h, h, h, h, 1e-6,
                              code, form, scale.data_ptr(), row_scales.data_ptr(), s)

        timings = {}
        touched = False
        try:
            plans = candidates(h // 16, variant == "fused") if h % 16 == 0 and not default_only \
                else []
            if form == capi.OUT_SAME and (tma or tma_only) and h % 8 == 0 and not default_only:
                plans = (plans if not tma_only else []) + tma_candidates(h, res_needed)

            for p in plans:
                touched = True
                capi.set_plan_override(p)
                try:
                    timings[p] = round(time_us(run, nsets), 2)
                except capi.HprnError:
                    pass  # plan not compiled for this variant (e.g. over its launch bound)
        finally:
            if touched:  # an override from HP_RMS_NORM_PLAN stays in force otherwise
                capi.set_plan_override(None)
        default = capi.plan(rows, h, code, xs[0].data_ptr(), rs[0].data_ptr()) \
            if variant == "fused" else "default"
        t_default = round(time_us(run, nsets), 2)
        best = min(timings, key=timings.get) if timings else default
        results[h] = {"default": default, "default_us": t_default,
                      "default_gbs": round(byt / t_default / 1e3, 1),
                      "best": best, "best_us": timings.get(best, t_default),
                      "plans": timings, "buffer_sets": nsets, "bytes_per_launch": byt}
        if copy:
            # torch's copy_ moving the same bytes (the kernel's reads into as
            # many bytes of writes), timed the same way.  The size is rounded
            # down to whole 4 KB: device-to-device copies of other sizes ran at
            # under half the bandwidth on B200.
            elems = byt // 4 // 2048 * 2048
            srcs = [torch.empty(elems, device=dev, dtype=tdt) for _ in range(nsets)]
            dsts = [torch.empty(elems, device=dev, dtype=tdt) for _ in range(nsets)]
            t_copy = round(time_us(lambda k, s: dsts[k].copy_(srcs[k]), nsets), 2)
            results[h]["copy_us"] = t_copy
            results[h]["copy_gbs"] = round(4 * elems / t_copy / 1e3, 1)
            del srcs, dsts
        del xs, rs, outs
        torch.cuda.empty_cache()
    return results


KNOBS = [f"default:pf{pf}:et{et}" for pf in (0, 1, 2, 3) for et in (0, 1, 2)]


def knob_sweep(a, reps: int = 3) -> None:
    """Times the default plan under every pair of launch knobs, each pair in
    its own process (HP_RMS_NORM_PLAN=default:pf<p>:et<e>), the pairs taken in
    turn `reps` times; prints the median per shape.  One process per pair
    because timings drift within a long-running process by more than the
    knobs' effect on short launches."""
    import os
    import subprocess
    import sys
    import tempfile

    runs = {k: [] for k in KNOBS}
    args = ["--rows", str(a.rows), "--hidden", a.hidden, "--dtype", a.dtype,
            "--variant", a.variant, "--default-only", "--no-tma"]
    if a.warm:
        args.append("--warm")
    with tempfile.TemporaryDirectory() as tmp:
        for rep in range(reps):
            for k in KNOBS:
                out = os.path.join(tmp, "r.json")
                env = dict(os.environ, HP_RMS_NORM_PLAN=k)
                subprocess.run([sys.executable, "-m", "hp_rms_norm_b200.tune", *args, "--json", out],
                               env=env, check=True, stdout=subprocess.DEVNULL)
                with open(out) as f:
                    runs[k].append(json.load(f))
    print(f"{a.variant} rows={a.rows} {'warm' if a.warm else 'cold'}: median us of {reps} processes")
    print(f"{'hidden':>7} " + " ".join(f"{k[8:]:>10}" for k in KNOBS))
    table = {}
    for h in a.hidden.split(","):
        meds = [sorted(r[h]["default_us"] for r in runs[k])[reps // 2] for k in KNOBS]
        table[h] = dict(zip(KNOBS, meds))
        print(f"{h:>7} " + " ".join(f"{m:>10.2f}" for m in meds))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(table, f, indent=1)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--hidden", default=",".join(str(h) for h in SWEEP))
    ap.add_argument("--dtype", choices=["bf16", "fp16"], default="bf16")
    ap.add_argument("--warm", action="store_true")
    ap.add_argument("--json", default=None)
    ap.add_argument("--variant", choices=list(VARIANTS), default="fused")
    ap.add_argument("--no-tma", action="store_true", help="leave out the TMA-staged plans")
    ap.add_argument("--tma-only", action="store_true", help="time only the TMA-staged plans")
    ap.add_argument("--isolated", action="store_true",
                    help="time single launches after an L2 flush instead of back-to-back graphs")
    ap.add_argument("--copy", action="store_true",
                    help="also time torch's copy_ of the same bytes, the same way")
    ap.add_argument("--default-only", action="store_true",
                    help="time only the built-in heuristic's plan (e.g. under an ncu capture)")
    ap.add_argument("--knobs", action="store_true",
                    help="time the default plan under every pair of launch knobs")
    a = ap.parse_args()
    if a.knobs:
        knob_sweep(a)
        return
    res = sweep(a.rows, [int(h) for h in a.hidden.split(",")], a.dtype, a.warm, a.variant,
                tma=not a.no_tma, tma_only=a.tma_only, isolated=a.isolated, copy=a.copy,
                default_only=a.default_only)
    print(f"{'hidden':>7} {'default plan':40} {'us':>8} {'GB/s':>8}   {'best plan':40} {'us':>8}"
          + (f" {'copy us':>8} {'copy GB/s':>9}" if a.copy else ""))
    for h, r in res.items():
        print(f"{h:>7} {r['default']:40} {r['default_us']:>8} {r['default_gbs']:>8}   "
              f"{r['best']:40} {r['best_us']:>8}"
              + (f" {r['copy_us']:>8} {r['copy_gbs']:>9}" if a.copy else ""))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
