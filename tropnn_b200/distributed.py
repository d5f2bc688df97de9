"""One-process-per-GPU data parallelism for the b200 layers.

The reference is single-device (no collective anywhere). Rows of a routed layer are
independent in forward and backward, so the layers scale by batch-row sharding: rank r
of W takes rows [r*N/W, (r+1)*N/W), keeps a full parameter replica, and after the
backward the parameter gradients are summed across ranks (NCCL all-reduce over
NVLink/NVSwitch for ``backend="nccl"``, gloo on CPU for tests) and divided by W, so
every rank holds the gradient of the global-batch mean loss.

Gradients are packed into flat buckets per dtype (``bucket_bytes`` each) so that a
layer with many small tensors costs a few collectives, while a large LUT gradient is
reduced in slices that can overlap with other work on the communication stream.
"""

from __future__ import annotations

from collections.abc import Iterable

import torch
import torch.distributed as dist
from torch import Tensor

__all__ = ["allreduce_gradients", "row_range", "shard_rows"]

DEFAULT_BUCKET_BYTES = 64 * 1024 * 1024


def row_range(rows: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous [start, stop) of ``rows`` owned by ``rank`` (balanced to within one row)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    base, extra = divmod(rows, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: Tensor, rank: int, world_size: int) -> Tensor:
    """This rank's row shard of ``t`` (rows along dim 0)."""
    start, stop = row_range(t.shape[0], rank, world_size)
    return t[start:stop]


def _buckets(grads: list[Tensor], bucket_bytes: int) -> list[list[Tensor]]:
    by_dtype: dict[torch.dtype, list[Tensor]] = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    out: list[list[Tensor]] = []
    for group in by_dtype.values():
        current: list[Tensor] = []
        size = 0
        for g in group:
            nbytes = g.numel() * g.element_size()
            if current and size + nbytes > bucket_bytes:
                out.append(current)
                current, size = [], 0
            current.append(g)
            size += nbytes
        if current:
            out.append(current)
    return out


def allreduce_gradients(
    params: Iterable[torch.nn.Parameter] | torch.nn.Module,
    *,
    group: dist.ProcessGroup | None = None,
    average: bool = True,
    bucket_bytes: int = DEFAULT_BUCKET_BYTES,
) -> int:
    """Sums (and by default averages) ``.grad`` of ``params`` across the process group.

    Parameters without a gradient are skipped on every rank alike (the set must match
    across ranks, as it does for replicas stepping the same layers). A single tensor
    larger than ``bucket_bytes`` is reduced in place in slices of that size. Returns the
    number of collectives issued.
    """
    if isinstance(params, torch.nn.Module):
        params = params.parameters()
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return 0
    world = dist.get_world_size(group)
    if world == 1:
        return 0
    calls = 0
    for bucket in _buckets(grads, bucket_bytes):
        if len(bucket) == 1:
            flat = bucket[0].view(-1)
            step = max(1, bucket_bytes // flat.element_size())
            for start in range(0, flat.numel(), step):
                piece = flat[start : start + step]
                dist.all_reduce(piece, op=dist.ReduceOp.SUM, group=group)
                calls += 1
                if average:
                    piece.div_(world)
            continue
        flat = torch.cat([g.reshape(-1) for g in bucket])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        calls += 1
        if average:
            flat.div_(world)
        offset = 0
        for g in bucket:
            n = g.numel()
            g.copy_(flat[offset : offset + n].view_as(g))
            offset += n
    return calls
