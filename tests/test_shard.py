"""Row sharding (the multi-GPU mode: rows split across ranks, no collective on
the data path), exercised with gloo ranks on CPU and the C oracle standing in
for each rank's GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hp_rms_norm_b200.shard import local_rows, row_range


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("rows", [0, 1, 7, 8, 33, 4096, 65536, 32769])
def test_row_range_partitions(rows, world):
    spans = [row_range(rows, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == rows
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_row_range_rejects_bad_splits():
    for args in ((4, 0, 0), (4, 2, 2), (4, 2, -1), (-1, 2, 0)):
        with pytest.raises(ValueError):
            row_range(*args)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, rows, hidden, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O

        g = np.random.default_rng(0)
        x = O.from_f32(O.BF16, g.standard_normal((rows, hidden)).astype(np.float32))
        r = O.from_f32(O.BF16, g.standard_normal((rows, hidden)).astype(np.float32))
        w = O.from_f32(O.BF16, (1 + 0.1 * g.standard_normal(hidden)).astype(np.float32))
        start, stop = local_rows(rows)
        out, res = O.fused_add_rms_norm(O.BF16, x[start:stop], w, r[start:stop], 1e-6)
        # Only the test gathers the shards (to check them); the product path has no collective.
        n = torch.tensor([stop - start])
        sizes = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
        dist.all_gather(sizes, n)
        cap = max(int(s) for s in sizes)
        pad = np.zeros((cap, hidden), dtype=np.uint16)
        pad[: stop - start] = out
        gathered = [torch.zeros(cap, hidden, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(pad.astype(np.int32)))
        if rank == 0:
            full = np.concatenate([g_.numpy()[: int(s)] for g_, s in zip(gathered, sizes)])
            want, _ = O.fused_add_rms_norm(O.BF16, x, w, r, 1e-6)
            np.save(os.path.join(out_dir, "ok.npy"), np.array([np.array_equal(full.astype(np.uint16), want)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_rows_reassemble_to_the_unsharded_result(tmp_path, world):
    mp.start_processes(_rank_main, args=(world, _free_port(), 37, 512, str(tmp_path)),
                       nprocs=world, start_method="spawn", join=True)
    assert bool(np.load(tmp_path / "ok.npy")[0])


def test_local_rows_without_process_group():
    assert local_rows(10) == (0, 10)
