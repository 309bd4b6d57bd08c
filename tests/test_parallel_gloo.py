"""The N>1 host logic (batch sharding, max-over-ranks timing) on CPU ranks (gloo)."""
import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp

from domino_b200.parallel import shard_rows


def test_shard_rows_cover_every_row_once():
    for total in range(0, 40):
        for world in range(1, 9):
            seen = []
            for r in range(world):
                s, n = shard_rows(total, world, r)
                seen.extend(range(s, s + n))
                assert n in (total // world, total // world + 1)
            assert seen == list(range(total))
    with pytest.raises(ValueError):
        shard_rows(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from domino_b200.parallel import all_gather_bytes, max_over_ranks, shard_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        start, count = shard_rows(7, world, rank)
        mx = max_over_ranks([10.0 * (rank + 1), -rank])
        blobs = all_gather_bytes(bytes([rank]) * 64)
        q.put((rank, start, count, mx, blobs))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_two_gloo_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(s, n) for _, s, n, _, _ in out] == [(0, 4), (4, 3)]
    for _, _, _, mx, blobs in out:
        assert mx == [20.0, 0.0]
        assert blobs == [bytes([0]) * 64, bytes([1]) * 64]
