"""Launch-plan sweep for the fused add + RMSNorm kernels.

    python -m hp_rms_norm_b200.tune [--rows 4096] [--hidden 1024,2048,...]
                                    [--dtype bf16|fp16] [--warm] [--json out.json]

Times every compiled launch plan that covers each requested shape (through
``hprn_set_plan_override``) and prints the fastest, next to the built-in
heuristic's choice.  Timing: a CUDA graph of back-to-back launches over
rotating buffer sets of at least 600 MB, so every launch reads cold data (or
one buffer set with ``--warm``), replayed three times after one warm replay.

This is how the heuristic in csrc/rms_norm.cu (``default_plan``) was fitted on
B200; rerun it to check the heuristic on another part or other shapes.
"""
from __future__ import annotations

import argparse
import json
import math

SWEEP = [1024 * i for i in range(1, 17)] + [20480, 24576, 28672, 32768]


def candidates(nvec: int) -> list[str]:
    """Plans (32-byte vectors) whose threads x vectors x CTAs cover nvec vectors."""
    out = []
    if nvec <= 128:
        for vpt in (1, 2, 3, 4):
            if vpt * 32 >= nvec > (vpt - 1) * 32:
                out += [f"warp:vec32:vpt{vpt}:tpr32:cluster1:rpc{r}" for r in (2, 4, 8)]
    for cl in (1, 2, 4, 8):
        for vpt in (1, 2, 3, 4, 6, 8):
            max_threads = 1024 if vpt <= 2 else (512 if vpt <= 4 else 256)
            sl = -(-nvec // cl)
            tpr = -(-(-(-sl // vpt)) // 32) * 32
            if tpr > max_threads or (tpr > 32 and (tpr - 32) * vpt >= sl):
                continue
            kind = "cta" if cl == 1 else "cluster"
            out.append(f"{kind}:vec32:vpt{vpt}:tpr{tpr}:cluster{cl}:rpc1")
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


def sweep(rows: int, hiddens: list[int], dtype: str = "bf16", warm: bool = False) -> dict:
    import torch

    from . import capi

    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    code = capi.DTYPE_BF16 if dtype == "bf16" else capi.DTYPE_FP16
    dev = torch.device("cuda", torch.cuda.current_device())
    results = {}
    for h in hiddens:
        set_bytes = rows * h * 2 * 2
        nsets = 1 if warm else max(3, min(512, math.ceil(600e6 / set_bytes)))
        xs = [torch.randn(rows, h, device=dev).to(tdt) for _ in range(nsets)]
        rs = [torch.randn(rows, h, device=dev).to(tdt) for _ in range(nsets)]
        w = (1 + 0.1 * torch.randn(h, device=dev)).to(tdt)
        byt = 4 * rows * h * 2 + 2 * h

        def run(k, s):
            capi.rms_norm(xs[k].data_ptr(), w.data_ptr(), rs[k].data_ptr(), rows, h, h, h, 1e-6,
                          code, s)

        timings = {}
        try:
            for p in candidates(h // 16) if h % 16 == 0 else []:
                capi.set_plan_override(p)
                timings[p] = round(graph_us(torch, run, nsets), 2)
        finally:
            capi.set_plan_override(None)
        default = capi.plan(rows, h, code, xs[0].data_ptr(), rs[0].data_ptr())
        t_default = round(graph_us(torch, run, nsets), 2)
        best = min(timings, key=timings.get) if timings else default
        results[h] = {"default": default, "default_us": t_default,
                      "default_gbs": round(byt / t_default / 1e3, 1),
                      "best": best, "best_us": timings.get(best, t_default),
                      "plans": timings, "buffer_sets": nsets}
        del xs, rs
        torch.cuda.empty_cache()
    return results


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--hidden", default=",".join(str(h) for h in SWEEP))
    ap.add_argument("--dtype", choices=["bf16", "fp16"], default="bf16")
    ap.add_argument("--warm", action="store_true")
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    res = sweep(a.rows, [int(h) for h in a.hidden.split(",")], a.dtype, a.warm)
    print(f"{'hidden':>7} {'default plan':40} {'us':>8} {'GB/s':>8}   {'best plan':40} {'us':>8}")
    for h, r in res.items():
        print(f"{h:>7} {r['default']:40} {r['default_us']:>8} {r['default_gbs']:>8}   "
              f"{r['best']:40} {r['best_us']:>8}")
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
