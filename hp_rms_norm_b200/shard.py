"""Row sharding for multi-GPU use.

Rows of the fused add + RMSNorm are independent and the weight is read-only,
so N GPUs split the rows and run the single-GPU path on their own block with
no collective at all: one process per GPU, each owning a contiguous block of
rows of its own tensors (bench.py's `--workload shard` and weak-scaling runs
are built on this).
"""
from __future__ import annotations


def row_range(rows: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of `rank`'s rows when `rows` are split over `world` ranks:
    contiguous blocks whose sizes differ by at most one, the larger blocks first."""
    if world < 1 or not 0 <= rank < world or rows < 0:
        raise ValueError(f"bad split: rows={rows} world={world} rank={rank}")
    base, extra = divmod(rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def local_rows(rows: int) -> tuple[int, int]:
    """row_range for this process, from torch.distributed (or the whole range
    when no process group is initialised)."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return row_range(rows, dist.get_world_size(), dist.get_rank())
    return 0, rows
