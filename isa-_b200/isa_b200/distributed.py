"""Data-parallel plumbing of the CIM operator: token sharding and one gradient
exchange per step.

The reference trains with DDP (``language/train.py:629,717``,
``vision/train.py:399``): tokens are sharded by a DistributedSampler and every
gradient, the threshold voltages included, is all-reduced.  The operator's
forward and dX are token-local, so the only exchange is the sum over tokens of
dVth (plus the scalar TIA / affine grads and any digital parameters).  Here that
is one flat-buffer all-reduce per step over NCCL (gloo on CPU), issued once the
backward has finished.
"""

from __future__ import annotations

from typing import Iterable, Optional

import torch
import torch.distributed as dist


def shard_rows(n: int, rank: int, world: int) -> slice:
    """Contiguous, balanced token range of ``rank`` (sizes differ by at most 1)."""
    lo = n * rank // world
    hi = n * (rank + 1) // world
    return slice(lo, hi)


def allreduce_gradients(params: Iterable[torch.nn.Parameter], group: Optional[dist.ProcessGroup] = None,
                        average: bool = True) -> int:
    """Sum (or average) the ``.grad`` of ``params`` over the group with a single
    all-reduce of one flat buffer per dtype.  Returns the bytes reduced."""
    world = dist.get_world_size(group)
    grads = [p.grad for p in params if p.grad is not None]
    total = 0
    by_dtype: dict[torch.dtype, list[torch.Tensor]] = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    for dtype, gs in by_dtype.items():
        flat = torch.cat([g.reshape(-1) for g in gs])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        if average and world > 1:
            flat.div_(world)
        off = 0
        for g in gs:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n
        total += flat.numel() * flat.element_size()
    return total
