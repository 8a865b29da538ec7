"""GPU parity of the fused add + RMSNorm kernels, called through the C ABI.

Bar (the task's): the updated residual is bit-exact to the 16-bit rounding of
the fp32 sum; the normalised output is within 1 ulp of T and within
atol 1e-2 / rtol 1e-2 of the fp32-accumulated reference (the C oracle at sizes
it finishes in seconds, a plain PyTorch fp32 reference at full BASELINE sizes).
"""
import os

import numpy as np
import pytest
import torch

from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import (DTYPES, bits, from_bits, make_inputs, torch_fp32_reference,
                               ulp_distance)
from tests.numerics import assert_bits_equal, assert_output_close

pytestmark = pytest.mark.gpu


def run_capi(x, w, r, eps):
    capi.rms_norm_tensors(x, w, r, eps)
    torch.cuda.synchronize()


def check_vs_oracle(x, w, r, eps, code, label, run=run_capi):
    xb, wb, rb = bits(x), bits(w), bits(r)
    want_out, want_res = O.fused_add_rms_norm(code, xb, wb, rb, eps, O.SS_UNROUNDED)
    run(x, w, r, eps)
    assert_bits_equal(bits(r), want_res, code, label=label + " residual")
    return assert_output_close(bits(x), want_out, code, label=label + " output")


def test_golden_fixtures(cuda, rms_golden):
    """Cases produced by the reference test's own formula (tests/golden)."""
    for case, c in rms_golden.items():
        tdtype, code = DTYPES[case[:4]]
        x = from_bits(c["x"], tdtype, cuda)
        r = from_bits(c["r"], tdtype, cuda)
        w = from_bits(c["w"], tdtype, cuda)
        run_capi(x, w, r, c["eps"])
        assert_bits_equal(bits(r), c["res"], code, label=case + " residual")
        assert_output_close(bits(x), c["out"], code, label=case)


DECODE_ROWS = [1, 7, 33, 128, 512]
DECODE_HIDDEN = [4096, 5120, 7168, 8192]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("hidden", DECODE_HIDDEN)
@pytest.mark.parametrize("rows", DECODE_ROWS)
def test_config2_decode_shapes(cuda, dtype, hidden, rows):
    tdtype, code = DTYPES[dtype]
    x, w, r, eps = make_inputs(rows, hidden, tdtype, "c2", seed=rows * 7 + hidden, device=cuda)
    check_vs_oracle(x, w, r, eps, code, f"{dtype} {rows}x{hidden}")


SWEEP = list(range(1024, 16384 + 1, 1024)) + [20480, 24576, 28672, 32768]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("rows,hidden", [(r, h) for r in (1, 7, 33, 128, 512, 513)
                                         for h in (1024, 1536, 2048)])
def test_small_batch_short_rows(cuda, dtype, rows, hidden):
    """Decode-sized batches of rows of 1024-2048 elements, config-2
    distributions: one CTA per row at 16-byte vectors up to 512 rows, the warp
    and CTA rules from 513."""
    tdtype, code = DTYPES[dtype]
    x, w, r, eps = make_inputs(rows, hidden, tdtype, "c2", seed=rows * 11 + hidden, device=cuda)
    check_vs_oracle(x, w, r, eps, code, f"{dtype} {rows}x{hidden} {capi.plan(rows, hidden)}")


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("hidden", SWEEP)
def test_hidden_sweep_vs_oracle(cuda, dtype, hidden):
    tdtype, code = DTYPES[dtype]
    x, w, r, eps = make_inputs(96, hidden, tdtype, "c0", seed=hidden, device=cuda)
    frac = check_vs_oracle(x, w, r, eps, code, f"{dtype} 96x{hidden}")
    assert frac < 0.05


def test_config0_full_size_vs_oracle(cuda):
    """4096 x 4096 bf16, seed 0, against the C oracle."""
    x, w, r, eps = make_inputs(4096, 4096, torch.bfloat16, "c0", seed=0, device=cuda)
    frac = check_vs_oracle(x, w, r, eps, O.BF16, "config0")
    assert frac < 0.01


@pytest.mark.parametrize("hidden", SWEEP)
def test_config1_full_batch_vs_torch_fp32(cuda, hidden):
    """BASELINE config 1 at its full batch of 4096 rows, against plain PyTorch fp32."""
    x, w, r, eps = make_inputs(4096, hidden, torch.bfloat16, "c0", seed=1000 + hidden, device=cuda)
    want_out, want_res = torch_fp32_reference(x, w, r, eps)
    run_capi(x, w, r, eps)
    assert torch.equal(r.view(torch.int16), want_res.view(torch.int16))
    assert int(ulp_distance(x, want_out).max()) <= 1
    torch.testing.assert_close(x.float(), want_out.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("rows,hidden", [(65536, 8192), (32768, 32768)])
def test_config4_full_shapes_vs_torch_fp32(cuda, rows, hidden):
    """BASELINE config 4's global batches at full size on one GPU (the
    multi-GPU mode runs the same kernel on each rank's block of these rows)."""
    x, w, r, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=rows, device=cuda)
    want_out, want_res = torch_fp32_reference(x, w, r, eps)
    run_capi(x, w, r, eps)
    assert torch.equal(r.view(torch.int16), want_res.view(torch.int16))
    assert int(ulp_distance(x, want_out).max()) <= 1
    del want_out, want_res


@pytest.mark.parametrize("rows,hidden,offset", [(2, 1 << 27, 0), (3, (1 << 26) + 7, 1)])
def test_longest_rows_vs_torch_fp32(cuda, rows, hidden, offset):
    """Rows of 2^26-2^27 elements (the clustered two-pass kernel, 32-bit vector
    indices far past any other case): 32-byte vectors, and an odd hidden size
    at a 2-byte offset (2-byte vectors, 2^26 of them per row)."""
    x, w, r, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=hidden, device=cuda)
    if offset:
        x = torch.empty(rows * hidden + offset, dtype=x.dtype, device=cuda)[offset:].view(rows, hidden).copy_(x)
    assert capi.plan(rows, hidden, capi.DTYPE_BF16, x.data_ptr(), r.data_ptr()).startswith("twopass")
    want_out, want_res = torch_fp32_reference(x, w, r, eps)
    run_capi(x, w, r, eps)
    assert torch.equal(r.view(torch.int16), want_res.view(torch.int16))
    assert int(ulp_distance(x, want_out).max()) <= 1
    del want_out, want_res


# Plans forced through the tuning hook: every kernel kind, vector width,
# vectors-per-thread and cluster size the library compiles.
FORCED = [
    (64, 512, "warp:vec32:vpt1:tpr32:cluster1:rpc1"),
    (65, 1024, "warp:vec32:vpt2:tpr32:cluster1:rpc4"),
    (67, 1536, "warp:vec32:vpt3:tpr32:cluster1:rpc8"),
    (63, 2048, "warp:vec32:vpt4:tpr32:cluster1:rpc2"),
    (9, 4096, "cta:vec32:vpt1:tpr256:cluster1:rpc1"),
    (9, 4096, "cta:vec32:vpt2:tpr128:cluster1:rpc1"),
    (9, 4096, "cta:vec32:vpt3:tpr96:cluster1:rpc1"),
    (9, 4096, "cta:vec32:vpt4:tpr64:cluster1:rpc1"),
    (9, 12288, "cta:vec32:vpt6:tpr128:cluster1:rpc1"),
    (9, 16384, "cta:vec32:vpt8:tpr128:cluster1:rpc1"),
    (9, 16384, "cluster:vec32:vpt2:tpr256:cluster2:rpc1"),
    (9, 32768, "cluster:vec32:vpt4:tpr128:cluster4:rpc1"),
    (9, 32768, "cluster:vec32:vpt2:tpr128:cluster8:rpc1"),
    (5, 13312, "cluster:vec32:vpt3:tpr160:cluster2:rpc1"),
    (9, 8192, "twopass:vec32:vpt4:tpr256:cluster1:rpc1"),
    (9, 8192, "cta:vec16:vpt4:tpr256:cluster1:rpc1"),
    (9, 8192, "cluster:vec8:vpt8:tpr128:cluster2:rpc1"),
    (9, 4096, "cta:vec4:vpt8:tpr256:cluster1:rpc1"),
    (9, 4096, "cluster:vec2:vpt8:tpr128:cluster4:rpc1"),
    (9, 4096, "twopass:vec2:vpt4:tpr512:cluster1:rpc1"),
    (9, 8192, "twopass:vec32:vpt4:tpr256:cluster2:rpc1"),
    (7, 20000, "twopass:vec32:vpt4:tpr128:cluster4:rpc1"),
    (5, 1 << 19, "twopass:vec32:vpt4:tpr512:cluster8:rpc1"),
    (9, 4097, "twopass:vec2:vpt4:tpr512:cluster4:rpc1"),
    (33, 256, "warp:vec16:vpt1:tpr32:cluster1:rpc8"),
    (33, 256, "warp:vec4:vpt4:tpr32:cluster1:rpc3"),
    (67, 64, "warp:vec32:vpt1:tpr4:cluster1:rpc64"),
    (5, 128, "warp:vec32:vpt2:tpr4:cluster1:rpc32"),
    (129, 256, "warp:vec32:vpt1:tpr16:cluster1:rpc16"),
    (33, 48, "warp:vec32:vpt3:tpr1:cluster1:rpc128"),
    (17, 512, "warp:vec32:vpt4:tpr8:cluster1:rpc32"),
    (9, 40, "warp:vec16:vpt2:tpr4:cluster1:rpc8"),
    (300, 16, "warp:vec32:vpt1:tpr1:cluster1:rpc256"),
]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("rows,hidden,plan", FORCED)
def test_every_plan_kind(cuda, dtype, rows, hidden, plan):
    tdtype, code = DTYPES[dtype]
    x, w, r, eps = make_inputs(rows, hidden, tdtype, "c0", seed=len(plan) + hidden, device=cuda)
    capi.set_plan_override(plan)
    try:
        check_vs_oracle(x, w, r, eps, code, plan)
    finally:
        capi.set_plan_override(None)


@pytest.mark.parametrize("hidden", [1, 2, 3, 7, 8, 15, 127, 4097, 5119, 12290, 20482])
def test_odd_hidden_sizes(cuda, hidden):
    x, w, r, eps = make_inputs(5, hidden, torch.float16, "c0", seed=hidden, device=cuda)
    check_vs_oracle(x, w, r, eps, O.FP16, f"hidden {hidden}")


def test_large_hidden_two_pass(cuda):
    """Rows past the register-resident kernels' reach (1M elements)."""
    hidden = 1 << 20
    assert capi.plan(2, hidden).startswith("twopass")
    x, w, r, eps = make_inputs(2, hidden, torch.bfloat16, "c0", seed=3, device=cuda)
    check_vs_oracle(x, w, r, eps, O.BF16, "1M")


def test_strided_rows_and_canaries(cuda):
    """Row strides differ from hidden and from each other; untouched columns,
    leading and trailing rows keep their sentinel bits."""
    rows, hidden = 37, 4096
    x0, w, r0, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=11, device=cuda)
    sentinel = -12345
    xbuf = torch.full((rows + 2, hidden + 64), sentinel, dtype=torch.int16, device=cuda)
    rbuf = torch.full((rows + 2, hidden + 128), sentinel, dtype=torch.int16, device=cuda)
    x = xbuf.view(torch.bfloat16)[1:-1, 16:16 + hidden]
    r = rbuf.view(torch.bfloat16)[1:-1, :hidden]
    x.copy_(x0)
    r.copy_(r0)
    want_out, want_res = O.fused_add_rms_norm(O.BF16, bits(x0), bits(w), bits(r0), eps)
    capi.rms_norm_tensors(x, w, r, eps)
    torch.cuda.synchronize()
    assert_bits_equal(bits(r), want_res, O.BF16, label="strided residual")
    assert_output_close(bits(x), want_out, O.BF16, label="strided output")
    xmask = torch.ones_like(xbuf, dtype=torch.bool)
    xmask[1:-1, 16:16 + hidden] = False
    rmask = torch.ones_like(rbuf, dtype=torch.bool)
    rmask[1:-1, :hidden] = False
    assert bool((xbuf[xmask] == sentinel).all())
    assert bool((rbuf[rmask] == sentinel).all())


def test_misaligned_pointers(cuda):
    """Tensors starting 2 bytes past an aligned address take the narrow path."""
    rows, hidden = 19, 2048
    x0, w0, r0, eps = make_inputs(rows, hidden, torch.float16, "c0", seed=5, device=cuda)
    xb = torch.empty(rows * hidden + 1, dtype=torch.float16, device=cuda)
    rb = torch.empty(rows * hidden + 1, dtype=torch.float16, device=cuda)
    wb = torch.empty(hidden + 1, dtype=torch.float16, device=cuda)
    x = xb[1:].view(rows, hidden)
    r = rb[1:].view(rows, hidden)
    w = wb[1:]
    x.copy_(x0)
    r.copy_(r0)
    w.copy_(w0)
    assert ":vec2:" in capi.plan(rows, hidden, capi.DTYPE_FP16, x.data_ptr(), r.data_ptr())
    check_vs_oracle(x, w, r, eps, O.FP16, "misaligned")


def test_special_values(cuda):
    rows, hidden = 4, 1024
    x = torch.zeros(rows, hidden, dtype=torch.float16, device=cuda)
    r = torch.zeros_like(x)
    w = torch.ones(hidden, dtype=torch.float16, device=cuda)
    x[1] = 60000.0  # fp16 residual overflows to inf -> output NaN, as in the oracle
    r[1] = 60000.0
    x[2, 5] = float("nan")
    x[3] = 1e-4
    check_vs_oracle(x, w, r, 1e-6, O.FP16, "special")


def test_torch_op_matches_capi(cuda):
    """The torch op (3-D input, the reference's Python API) gives the C ABI's bits."""
    import hp_rms_norm_b200

    x, w, r, eps = make_inputs(6 * 85, 5120, torch.bfloat16, "c0", seed=21, device=cuda)
    x3, r3 = x.clone().view(6, 85, 5120), r.clone().view(6, 85, 5120)
    hp_rms_norm_b200.hp_rms_norm(x3, w, r3, eps)
    capi.rms_norm_tensors(x, w, r, eps)
    torch.cuda.synchronize()
    assert torch.equal(x3.view(-1, 5120).view(torch.int16), x.view(torch.int16))
    assert torch.equal(r3.view(-1, 5120).view(torch.int16), r.view(torch.int16))


def test_torch_op_argument_errors(cuda):
    import hp_rms_norm_b200

    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    r = torch.zeros_like(x)
    w = torch.ones(64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="dtype must be kFloat16 or kBFloat16"):
        hp_rms_norm_b200.hp_rms_norm(x.float(), w.float(), r.float(), 1e-6)
    with pytest.raises(RuntimeError, match="input.size\\(-1\\) == hidden_dim"):
        hp_rms_norm_b200.hp_rms_norm(x, w[:32], r, 1e-6)
    with pytest.raises(RuntimeError, match="input.dim\\(\\) >= 2"):
        hp_rms_norm_b200.hp_rms_norm(x[0], w, r[0], 1e-6)
    with pytest.raises(RuntimeError, match="same dtype"):
        hp_rms_norm_b200.hp_rms_norm(x, w.half(), r, 1e-6)
    with pytest.raises(RuntimeError, match="stride\\(-1\\) == 1"):
        hp_rms_norm_b200.hp_rms_norm(x.t().contiguous().t(), w, r, 1e-6)
    with pytest.raises(RuntimeError, match="overlap"):
        hp_rms_norm_b200.hp_rms_norm(x, w, x, 1e-6)


def test_deterministic_and_graph_capturable(cuda):
    x0, w, r0, eps = make_inputs(512, 8192, torch.bfloat16, "c0", seed=9, device=cuda)
    x1, r1 = x0.clone(), r0.clone()
    capi.rms_norm_tensors(x1, w, r1, eps)
    x2, r2 = x0.clone(), r0.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        capi.rms_norm_tensors(x2, w, r2, eps, stream=s.cuda_stream)
    x2.copy_(x0)
    r2.copy_(r0)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(x1.view(torch.int16), x2.view(torch.int16))
    assert torch.equal(r1.view(torch.int16), r2.view(torch.int16))


def test_concurrent_host_threads(cuda):
    """Eight host threads call the C ABI at once, each on its own stream with
    its own shape (kernels whose occupancy the per-device cache may not hold
    yet are launched concurrently); every result equals the same call made
    alone afterwards."""
    import threading

    shapes = [(257, 1024), (300, 2560), (129, 4096), (64, 7168), (96, 12288), (40, 20480),
              (16, 40960), (8, 1 << 17)]
    inputs = [make_inputs(rows, hidden, torch.bfloat16, "c0", seed=rows + hidden, device=cuda)
              for rows, hidden in shapes]
    torch.cuda.synchronize()
    got = [None] * len(shapes)
    errors = []

    def work(k):
        try:
            x0, w, r0, eps = inputs[k]
            s = torch.cuda.Stream(device=cuda)
            with torch.cuda.stream(s):
                x, r = x0.clone(), r0.clone()
                for _ in range(3):  # same inputs each time: the last call's result is compared
                    x.copy_(x0)
                    r.copy_(r0)
                    capi.rms_norm_tensors(x, w, r, eps, stream=s.cuda_stream)
            s.synchronize()
            got[k] = (x, r)
        except Exception as e:  # reported below, on the main thread
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(k,)) for k in range(len(shapes))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    want = []
    for x0, w, r0, eps in inputs:
        x, r = x0.clone(), r0.clone()
        capi.rms_norm_tensors(x, w, r, eps)
        want.append((x, r))
    torch.cuda.synchronize()
    for (wx, wr), (gx, gr) in zip(want, got):
        assert torch.equal(wx.view(torch.int16), gx.view(torch.int16))
        assert torch.equal(wr.view(torch.int16), gr.view(torch.int16))


def test_first_calls_inside_graph_capture(cuda):
    """A process whose first calls of each kernel shape happen inside a CUDA
    graph capture (the library queries a kernel's occupancy once per device
    on its first launch, to size the L2 prefetch) captures, replays and gives
    the bits of eager launches (tests/graph_first_call_worker.py, run in a
    fresh process so no kernel shape has been launched before)."""
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = subprocess.run([sys.executable, os.path.join(root, "tests", "graph_first_call_worker.py")],
                       cwd=root, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-3000:]


REF_SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                      "libhp_rms_norm_ref.so")


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("hidden", [1024, 4096, 8192, 12288, 13312, 16384, 20480])
def test_matches_reference_cuda_kernel(cuda, hidden):
    """Same inputs through the reference's own CUDA kernel (compiled from its
    sources): residual bit-exact, output within 1 ulp."""
    ref = O.ReferenceKernels(REF_SO)
    x, w, r, eps = make_inputs(512, hidden, torch.bfloat16, "c0", seed=hidden + 1, device=cuda)
    xr, rr = x.clone(), r.clone()
    ref.rms_norm(xr, w, rr, eps)
    run_capi(x, w, r, eps)
    assert torch.equal(r.view(torch.int16), rr.view(torch.int16))
    assert int(ulp_distance(x, xr).max()) <= 1


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_reference_test_grid_matches_reference_cuda_kernel(cuda, dtype):
    """The reference test's own grid (hidden 128..32768 in steps of 128, a
    random token count of 1..4096 per shape, inputs and weight ~ N(0, 0.1),
    eps = bf16 epsilon; test/test_hp_rms_norm.py:49-58), seeded, up to hidden
    24448 (the reference's build on this toolchain rejects >= 24576), through
    the reference's own CUDA kernel and this library: residual bit-exact,
    output within 1 ulp at every shape."""
    tdtype, _ = DTYPES[dtype]
    ref = O.ReferenceKernels(REF_SO)
    rng = np.random.default_rng(2024 if dtype == "bf16" else 2025)
    worst, differing, total = 0, 0, 0
    for hidden in range(128, 24448 + 1, 128):
        rows = int(rng.integers(1, 4097))
        g = torch.Generator(device=cuda).manual_seed(hidden)  # the "rt" distribution, on the device
        x = (0.1 * torch.randn(rows, hidden, generator=g, device=cuda)).to(tdtype)
        r = (0.1 * torch.randn(rows, hidden, generator=g, device=cuda)).to(tdtype)
        w = (0.1 * torch.randn(hidden, generator=g, device=cuda)).to(tdtype)
        eps = float(torch.finfo(torch.bfloat16).eps)
        xr, rr = x.clone(), r.clone()
        ref.rms_norm(xr, w, rr, eps)
        run_capi(x, w, r, eps)
        assert torch.equal(r.view(torch.int16), rr.view(torch.int16)), f"residual differs at {rows}x{hidden}"
        d = ulp_distance(x, xr)
        m = int(d.max())
        assert m <= 1, f"output {m} ulp from the reference kernel at {rows}x{hidden}"
        worst = max(worst, m)
        differing += int((d > 0).sum())
        total += d.numel()
    # Outputs that differ by one ulp come from the sum of squares' order
    # (a different reduction tree); they stay rare.
    assert differing / total < 0.01, differing / total


@pytest.mark.parametrize("hidden", [1024, 4096, 20480, 65536])
def test_pdl_chains_match_plain_launches(cuda, hidden):
    """Back-to-back dependent launches (each call reads the previous call's
    output, then ReLU reads the last output) give the same bits with
    programmatic dependent launch as with plain launches, eagerly and inside a
    CUDA graph."""
    rows = 64 if hidden > 32768 else 512
    x0, w, r0, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=hidden + 7, device=cuda)

    def chain(x, r, out, flags, stream):
        for _ in range(3):
            capi.rms_norm_tensors(x, w, r, eps, stream=stream, flags=flags)
        capi.relu_tensors(out, x, stream=stream, flags=flags)

    results = []
    for flags in (0, capi.LAUNCH_PDL):
        x, r, out = x0.clone(), r0.clone(), torch.empty_like(x0)
        chain(x, r, out, flags, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        results.append((x, r, out))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    xg, rg, og = x0.clone(), r0.clone(), torch.empty_like(x0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        chain(xg, rg, og, capi.LAUNCH_PDL, s.cuda_stream)
    xg.copy_(x0)
    rg.copy_(r0)
    g.replay()
    torch.cuda.synchronize()
    results.append((xg, rg, og))
    for got in results[1:]:
        for a, b in zip(results[0], got):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))


KNOBS = [f"default:pf{pf}:et{et}" for pf in (0, 1, 2, 3) for et in (0, 1, 2)]


@pytest.mark.parametrize("knobs", KNOBS)
@pytest.mark.parametrize("rows,hidden", [(512, 1024), (600, 4096), (300, 24576), (64, 65536),
                                         (4, 1 << 18)])
def test_launch_knobs_keep_results(cuda, knobs, rows, hidden):
    """The launch knobs only move work in time: an L2 prefetch issued before
    the programmatic-launch wait (on lines the preceding call is still
    writing), and the point where dependents are triggered.  Dependent chains
    under every pair give the bits of plain launches (warp, CTA, cluster and
    two-pass kernels; grids of more than one wave)."""
    x0, w, r0, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=hidden + 11, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream

    def chain(flags):
        x, r, out = x0.clone(), r0.clone(), torch.empty_like(x0)
        for _ in range(3):
            capi.rms_norm_tensors(x, w, r, eps, stream=stream, flags=flags)
        capi.relu_tensors(out, x, stream=stream, flags=flags)
        torch.cuda.synchronize()
        return x, r, out

    want = chain(0)
    capi.set_plan_override(knobs)
    try:
        assert capi.plan(rows, hidden).endswith(knobs[7:])
        got = chain(capi.LAUNCH_PDL)
    finally:
        capi.set_plan_override(None)
    for a, b in zip(want, got):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_launch_flags_validated(cuda):
    x, w, r, eps = make_inputs(4, 256, torch.bfloat16, "c0", seed=1, device=cuda)
    with pytest.raises(capi.HprnError, match="unknown launch flags"):
        capi.rms_norm_tensors(x, w, r, eps, flags=0x80)


def test_torch_compile_fullgraph(cuda):
    """The mutation-annotated schemas and Meta kernels let torch.compile trace
    the ops with fullgraph=True; results match eager bit for bit."""
    import hp_rms_norm_b200

    def block(x, r, w, out):
        hp_rms_norm_b200.hp_rms_norm(x, w, r, 1e-6)
        hp_rms_norm_b200.relu(out, x)
        return out * 2

    x0, w, r0, _ = make_inputs(64, 4096, torch.bfloat16, "c0", seed=17, device=cuda)
    xe, re, oe = x0.clone(), r0.clone(), torch.empty_like(x0)
    want = block(xe, re, w, oe)
    compiled = torch.compile(block, fullgraph=True)
    xc, rc, oc = x0.clone(), r0.clone(), torch.empty_like(x0)
    got = compiled(xc, rc, w, oc)
    torch.cuda.synchronize()
    for a, b in ((want, got), (xe, xc), (re, rc), (oe, oc)):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
