"""Request-batch data parallelism for the draft step (one process per GPU).

Sequences are independent (the reference's block loop runs one sequence,
code/dflash.py:322-325, and its benchmark stripes requests over ranks,
code/benchmark.py:179), so ranks split the request batch and run the draft
step with no collective on the data path.  The only communication is for
reporting: the slowest rank's time.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple


def shard_rows(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous near-equal split of ``global_batch`` rows: (first row, row count) of ``rank``.

    The first ``global_batch % world`` ranks take one extra row; a rank may get
    zero rows when ``global_batch < world``.
    """
    if world < 1 or not 0 <= rank < world or global_batch < 0:
        raise ValueError(f"bad shard request: batch={global_batch} world={world} rank={rank}")
    base, extra = divmod(global_batch, world)
    count = base + (1 if rank < extra else 0)
    start = rank * base + min(rank, extra)
    return start, count


def max_over_ranks(values: Sequence[float], device=None) -> List[float]:
    """Element-wise maximum of ``values`` over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def all_gather_bytes(blob: bytes) -> List[bytes]:
    """Every rank's ``blob`` (e.g. a 64-byte CUDA IPC handle), in rank order."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [bytes(blob)]
    out: List[bytes] = [b""] * dist.get_world_size()
    dist.all_gather_object(out, bytes(blob))
    return out
