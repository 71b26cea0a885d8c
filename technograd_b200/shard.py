"""Data-parallel sharding of rows / sequences over ranks (one process per GPU).

Rows and sequences are independent units (src/main.c:216-242 runs each through
its own arena), so rank r of W takes the contiguous shard [r*R/W, (r+1)*R/W)
and computes with no exchange. The one exchange is the final gather of every
rank's output in input order. Timing across ranks is the max over ranks.

The helpers work on either backend: NCCL (device tensors) or gloo (host
tensors, used by the multi-process CPU tests).
"""
from __future__ import annotations

import numpy as np


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous shard of `total` units for `rank` of `world`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request: total {total}, world {world}, rank {rank}")
    return total * rank // world, total * (rank + 1) // world


def _device():
    import torch
    import torch.distributed as dist
    return torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")


def max_over_ranks(x: float, world: int) -> float:
    """The largest of every rank's `x` (a time), on every rank."""
    if world == 1:
        return float(x)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_in_order(local: np.ndarray, total: int, world: int, rank: int, dst: int = 0):
    """Every rank's shard of a [total, ...] result, concatenated in input order on `dst`
    (None on the other ranks). Shards are the shard_range() blocks, so their sizes are
    known everywhere and no size exchange is needed."""
    local = np.ascontiguousarray(local)
    if world == 1:
        return local
    import torch
    import torch.distributed as dist
    lo, hi = shard_range(total, world, rank)
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank}: shard has {local.shape[0]} rows, expected {hi - lo}")
    dev = _device()
    tail = local.shape[1:]
    biggest = max(shard_range(total, world, r)[1] - shard_range(total, world, r)[0] for r in range(world))
    buf = torch.zeros((biggest, *tail), dtype=torch.from_numpy(local[:0]).dtype, device=dev)
    buf[:local.shape[0]] = torch.from_numpy(local).to(dev)
    parts = [torch.empty_like(buf) for _ in range(world)] if rank == dst else None
    dist.gather(buf, parts, dst=dst)
    if rank != dst:
        return None
    out = []
    for r in range(world):
        a, b = shard_range(total, world, r)
        out.append(parts[r][:b - a].cpu().numpy())
    return np.concatenate(out, axis=0)
