"""Two devices in one process (runs only where at least two GPUs are visible):
the torch ops follow the tensors' device whatever the current device is (the
reference launches on the current device instead, hp_rms_norm.cu:27), and the
C ABI's per-device caches (device attributes, TMA-staged plan occupancy) serve
each device its own entry.  Rows sharded over the devices with
shard.row_range give the single-device result bit for bit."""
import pytest
import torch

import hp_rms_norm_b200 as H
from hp_rms_norm_b200 import capi, shard
from oracle import oracle as O
from tests.gpu_helpers import bits, make_inputs
from tests.numerics import assert_bits_equal, assert_output_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def two_devices(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    return torch.device("cuda", 0), torch.device("cuda", 1)


def test_torch_op_runs_on_the_tensors_device(two_devices):
    d0, d1 = two_devices
    x0, w0, r0, eps = make_inputs(257, 4096, torch.bfloat16, "c0", seed=21, device="cpu")
    want_out, want_res = O.fused_add_rms_norm(O.BF16, bits(x0), bits(w0), bits(r0), eps)
    x, w, r = x0.to(d1), w0.to(d1), r0.to(d1)
    with torch.cuda.device(d0):  # current device differs from the tensors'
        H.hp_rms_norm(x, w, r, eps)
        out = torch.empty_like(x)
        H.relu(out, x)
    torch.cuda.synchronize(d1)
    assert_bits_equal(bits(r), want_res, O.BF16, label="residual on cuda:1")
    assert_output_close(bits(x), want_out, O.BF16, label="output on cuda:1")
    assert torch.equal(out, torch.relu(x))


def test_c_abi_per_device_caches(two_devices):
    """The same TMA-staged plan on both devices, in alternation, then the
    default plan: every call matches the oracle."""
    x0, w0, r0, eps = make_inputs(1000, 2048, torch.float16, "c0", seed=22, device="cpu")
    want_out, want_res = O.fused_add_rms_norm(O.FP16, bits(x0), bits(w0), bits(r0), eps)
    for plan in ("tma:vec16:vpt2:tpr128:cluster1:rpc4", None):
        capi.set_plan_override(plan)
        try:
            for dev in (*two_devices, *two_devices):
                with torch.cuda.device(dev):
                    capi.wait_timeouts(reset=True)
                    x, w, r = x0.to(dev), w0.to(dev), r0.to(dev)
                    capi.rms_norm_tensors(x, w, r, eps)
                    torch.cuda.synchronize(dev)
                    assert capi.wait_timeouts() == 0
                    label = f"{plan or 'default'} on {dev}"
                    assert_bits_equal(bits(r), want_res, O.FP16, label=label + " residual")
                    assert_output_close(bits(x), want_out, O.FP16, label=label)
        finally:
            capi.set_plan_override(None)


def test_rows_sharded_over_devices_match_one_device(two_devices):
    rows, hidden = 4099, 8192
    x0, w0, r0, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=23, device=two_devices[0])
    x_one, r_one = x0.clone(), r0.clone()
    H.hp_rms_norm(x_one, w0, r_one, eps)
    world = len(two_devices)
    parts = []
    for rank, dev in enumerate(two_devices):
        a, b = shard.row_range(rows, world, rank)
        x, w, r = (t.to(dev, copy=True) for t in (x0[a:b], w0, r0[a:b]))
        H.hp_rms_norm(x, w, r, eps)
        parts.append((x, r))
    for dev in two_devices:
        torch.cuda.synchronize(dev)
    x_cat = torch.cat([p[0].to(two_devices[0]) for p in parts])
    r_cat = torch.cat([p[1].to(two_devices[0]) for p in parts])
    assert torch.equal(x_cat.view(torch.int16), x_one.view(torch.int16))
    assert torch.equal(r_cat.view(torch.int16), r_one.view(torch.int16))


def test_rows_sharded_over_ranks_under_torchrun(two_devices, tmp_path):
    """The same split as above in bench.py's multi-GPU layout: two processes
    started by torchrun, one per GPU, each running its own block of rows
    (tests/shard_rank_worker.py).  The blocks put together equal the
    one-device result bit for bit."""
    import os
    import socket
    import subprocess
    import sys

    import numpy as np

    from tests import shard_rank_worker as W

    x0, w0, r0, eps = make_inputs(W.ROWS, W.HIDDEN, torch.bfloat16, "c0", seed=W.SEED, device="cpu")
    x, w, r = x0.to(two_devices[0]), w0.to(two_devices[0]), r0.to(two_devices[0])
    H.hp_rms_norm(x, w, r, eps)
    torch.cuda.synchronize(two_devices[0])
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES=os.environ.get(
        "CUDA_VISIBLE_DEVICES", "0,1"))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(root, "tests", "shard_rank_worker.py"), str(tmp_path)]
    p = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    parts = [np.load(tmp_path / f"rank{k}.npz") for k in range(2)]
    assert int(parts[0]["start"]) == 0 and int(parts[0]["stop"]) == int(parts[1]["start"])
    assert int(parts[1]["stop"]) == W.ROWS
    assert np.array_equal(np.concatenate([q["res"] for q in parts]), bits(r))
    assert np.array_equal(np.concatenate([q["out"] for q in parts]), bits(x))
