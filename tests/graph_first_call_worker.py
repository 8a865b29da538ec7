"""Worker of tests/test_gpu_rms_norm.py::test_first_calls_inside_graph_capture,
run in a fresh process so that the library's first call of each kernel shape
(which queries the kernel's occupancy once per device and caches it) happens
while a CUDA graph is being captured.  Captures one call of each form and
launch kind, replays the graph, then runs the same calls eagerly and checks
the bits agree.  Exits non-zero on any difference.  Not a test module itself."""
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from hp_rms_norm_b200 import capi  # noqa: E402


def main() -> int:
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    eps = 1e-6
    # (rows, hidden): warp rows, CTA rows (one and two vectors per thread), a
    # cluster, two passes.
    shapes = [(300, 1024), (600, 4096), (300, 24576), (16, 65536), (4, 1 << 18)]
    base = []
    for rows, hidden in shapes:
        x = torch.randn(rows, hidden, generator=g, device=dev).to(torch.bfloat16)
        r = torch.randn(rows, hidden, generator=g, device=dev).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).to(torch.bfloat16)
        base.append((x, r, w))
    nv_x = torch.randn(256, 8192, generator=g, device=dev).to(torch.bfloat16)
    nv_w = (1 + 0.1 * torch.randn(8192, generator=g, device=dev)).to(torch.bfloat16)
    gs = torch.tensor([336.0], device=dev)
    act_in = torch.randn(64, 2 * 4096, generator=g, device=dev).to(torch.bfloat16)

    def run(bufs, stream):
        for (x, r, w) in bufs["rms"]:
            capi.rms_norm_tensors(x, w, r, eps, stream=stream)
        capi.rms_norm_nvfp4_tensors(bufs["nv_out"], bufs["nv_sf"], nv_x, nv_w, None, eps, gs,
                                    stream=stream)
        capi.relu_tensors(bufs["relu"], base[1][0], stream=stream)
        capi.act_and_mul_tensors(bufs["act"], act_in, capi.ACT_GELU, stream=stream)

    def fresh():
        return {"rms": [(x.clone(), r.clone(), w) for (x, r, w) in base],
                "nv_out": torch.zeros(256, 4096, dtype=torch.uint8, device=dev),
                "nv_sf": torch.zeros(256, 512, dtype=torch.uint8, device=dev),
                "relu": torch.zeros_like(base[1][0]),
                "act": torch.zeros(64, 4096, dtype=torch.bfloat16, device=dev)}

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graphed = fresh()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):  # the library's first calls in this process
        run(graphed, s.cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    eager = fresh()
    run(eager, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    bad = 0
    for (xa, ra, _), (xb, rb, _) in zip(graphed["rms"], eager["rms"]):
        bad += not torch.equal(xa.view(torch.int16), xb.view(torch.int16))
        bad += not torch.equal(ra.view(torch.int16), rb.view(torch.int16))
    for k in ("nv_out", "nv_sf", "relu", "act"):
        a, b = graphed[k], eager[k]
        bad += not torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    print("differences:", bad)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
