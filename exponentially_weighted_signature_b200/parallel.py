"""Data parallelism for the EWS hot path: batch sharding and the one parameter-gradient allreduce.

Samples are independent, so the scan shards by batch with no collective; after the backward the
parameter gradients (generator, lift, clock parameters) are summed across ranks with a single NCCL
allreduce of one flat bucket (the reference runs on one device and has no such layer).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int):
    """[start, stop) of this rank's contiguous batch shard; every rank gets total // world (+1 for the
    first total % world ranks)."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def allreduce_gradients(params, group=None, average: bool = False) -> None:
    """Sums (or averages) the .grad of ``params`` across the process group in one collective."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    if average:
        flat /= dist.get_world_size(group)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off : off + n].view_as(g))
        off += n
