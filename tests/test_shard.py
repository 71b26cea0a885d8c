"""Host-side data-parallel logic (technograd_b200.shard) on 2 gloo ranks (CPU).

Shards are contiguous and cover every unit once, times combine as the max over
ranks, and the output gather reassembles every rank's rows in input order, for
even and uneven splits."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from technograd_b200.shard import gather_in_order, max_over_ranks, shard_range


def test_shard_range_partitions():
    for total in (0, 1, 7, 64, 2048, 2049):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        res = {"max": max_over_ranks(1.5 + rank, world)}
        for total in (8, 7, 1):
            full = np.arange(total * 3, dtype=np.float32).reshape(total, 3) * 0.5
            lo, hi = shard_range(total, world, rank)
            got = gather_in_order(full[lo:hi], total, world, rank)
            res[f"f{total}"] = None if got is None else got.tolist()
            steps = (np.arange(total, dtype=np.int32) % 5).reshape(total, 1)
            got = gather_in_order(steps[lo:hi], total, world, rank)
            res[f"i{total}"] = None if got is None else got.tolist()
        q.put((rank, res))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert out[r]["max"] == 2.5
    for total in (8, 7, 1):
        full = np.arange(total * 3, dtype=np.float32).reshape(total, 3) * 0.5
        assert np.array_equal(np.array(out[0][f"f{total}"], np.float32), full)
        assert np.array_equal(np.array(out[0][f"i{total}"]), (np.arange(total) % 5).reshape(total, 1))
        assert out[1][f"f{total}"] is None
