"""One rank of the two-rank sharding test (tests/test_gpu_multi_device.py::
test_rows_sharded_over_ranks_under_torchrun), launched the way bench.py runs
under torchrun: one process per GPU, rank and device from the environment,
an NCCL process group used only for barriers.  Each rank takes its block of
rows (shard.local_rows), runs hp_rms_norm on its own GPU and writes the
resulting bits to <outdir>/rank<r>.npz.  Not a test module itself."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import hp_rms_norm_b200 as H  # noqa: E402
from hp_rms_norm_b200 import shard  # noqa: E402
from tests.gpu_helpers import bits, make_inputs  # noqa: E402

ROWS, HIDDEN, SEED = 4099, 8192, 23


def main(outdir: str) -> None:
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        x0, w0, r0, eps = make_inputs(ROWS, HIDDEN, torch.bfloat16, "c0", seed=SEED, device="cpu")
        a, b = shard.local_rows(ROWS)
        x, w, r = x0[a:b].to(dev), w0.to(dev), r0[a:b].to(dev)
        H.hp_rms_norm(x, w, r, eps)
        torch.cuda.synchronize(dev)
        np.savez(os.path.join(outdir, f"rank{dist.get_rank()}.npz"), start=a, stop=b,
                 out=bits(x), res=bits(r))
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
