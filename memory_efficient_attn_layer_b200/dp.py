"""Data-parallel gradient exchange for the block.

The block's batch shards across ranks by sequence (one process per GPU); the
only exchange is the all-reduce of the five weight gradients (Wq, Wk, Wv, Wg,
Wo) after each backward.  They are exchanged as one coalesced fp32 bucket (one
collective instead of five, and no bf16 rounding inside the sum), then written
back to each ``.grad`` in its own dtype.  The rotary tables are buffers, not
parameters, so their gradients are not exchanged.
"""
from __future__ import annotations

from typing import Iterable, Optional

import torch
import torch.distributed as dist


def allreduce_grads(params: Iterable[torch.Tensor], group: Optional[dist.ProcessGroup] = None,
                    average: bool = True) -> None:
    """All-reduce the ``.grad`` of every tensor in ``params`` across ``group``.

    Tensors without a gradient are skipped (every rank must pass the same
    parameters with the same gradient presence, as for any collective).  With
    ``average`` the sum is divided by the group size (the mean gradient over
    the global batch when every rank's loss is a mean over its own shard)."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    world = dist.get_world_size(group)
    bucket = torch.cat([g.reshape(-1).to(torch.float32) for g in grads])
    dist.all_reduce(bucket, group=group)
    if average and world > 1:
        bucket.div_(world)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(bucket[off:off + n].view_as(g))
        off += n
