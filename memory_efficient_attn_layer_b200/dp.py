"""Data-parallel gradient exchange for the block.

The block's batch shards across ranks by sequence (one process per GPU); the
only exchange is the all-reduce of the five weight gradients (Wq, Wk, Wv, Wg,
Wo).  They are exchanged in fp32 (no bf16 rounding inside the sum) and written
back to each gradient in its own dtype.  The rotary tables are buffers, not
parameters, so their gradients are not exchanged.

Two ways to run it:

* ``allreduce_grads(params)`` after ``loss.backward()``: one coalesced fp32
  bucket, one collective, nothing overlapped.
* ``with overlap_grad_allreduce(group): y = block(x); ...; loss.backward()``:
  every ``FusedAttentionFunction`` forward run inside the context tags its
  node, and that node's backward exchanges its own weight gradients while the
  rest of its backward still runs.  The library records an event as soon as
  the fp32 o_proj gradient is final (before the attention backward) and
  another when the q/k/v/g gradients are (before the input-gradient GEMM);
  the all-reduce of each part starts at its event on a side stream, and the
  caller's stream waits for the exchange only where the backward returns.  The
  gradients handed back to autograd are already the group mean (or sum), so
  ``allreduce_grads`` must not be called for those weights as well.

A third way replaces the exchange: ``optim.ShardedAdamW`` registers itself as
a gradient sink (``register_grad_sink``).  A block whose five weights it owns
writes its fp32 weight gradients straight into the optimizer's buffer, and the
optimizer reduce-scatters them in ``step()``.  The sink takes precedence over
an enclosing ``overlap_grad_allreduce``.
"""
from __future__ import annotations

import contextlib
import weakref
from typing import Callable, Iterable, Optional

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


def reduce_weight_grads(buf: torch.Tensor, n_qkvg: int, group: Optional[dist.ProcessGroup] = None,
                        average: bool = True, before_qkvg: Optional[Callable[[], None]] = None) -> None:
    """All-reduce the block's fp32 weight-gradient buffer in the order the
    backward finishes it: ``buf[n_qkvg:]`` (Wo) first, then ``buf[:n_qkvg]``
    (Wq, Wk, Wv, Wg), with ``before_qkvg`` run between the two (the overlapped
    path makes the side stream wait for the second readiness event there).
    Every rank issues the same two collectives in the same order."""
    dist.all_reduce(buf[n_qkvg:], group=group)
    if before_qkvg is not None:
        before_qkvg()
    dist.all_reduce(buf[:n_qkvg], group=group)
    if average and dist.get_world_size(group) > 1:
        buf.div_(dist.get_world_size(group))


_SIDE_STREAMS = {}


def side_stream(device: torch.device) -> "torch.cuda.Stream":
    """The per-device stream the overlapped exchange runs on.  High priority:
    the collective's kernels are scheduled ahead of the block's own grids as
    SMs free up."""
    s = _SIDE_STREAMS.get(device.index)
    if s is None:
        s = torch.cuda.Stream(device=device, priority=-1)
        _SIDE_STREAMS[device.index] = s
    return s


class GradExchange:
    """Settings of one overlapped exchange context."""

    def __init__(self, group: Optional[dist.ProcessGroup] = None, average: bool = True):
        self.group = group
        self.average = average


_ACTIVE: Optional[GradExchange] = None


def active_exchange() -> Optional[GradExchange]:
    """The exchange a forward run now should tag its node with (None outside
    an ``overlap_grad_allreduce`` context or with a group of one rank)."""
    ex = _ACTIVE
    if ex is None or not dist.is_available() or not dist.is_initialized():
        return None
    if dist.get_world_size(ex.group) <= 1:
        return None
    return ex


@contextlib.contextmanager
def overlap_grad_allreduce(group: Optional[dist.ProcessGroup] = None, average: bool = True):
    """Forwards of the block run inside this context exchange their weight
    gradients across ``group`` during their own backward (see the module
    docstring).  The backward itself may run after the context has closed."""
    global _ACTIVE
    prev = _ACTIVE
    _ACTIVE = GradExchange(group, average)
    try:
        yield _ACTIVE
    finally:
        _ACTIVE = prev


_SINKS: list = []


def register_grad_sink(sink) -> None:
    """Registers an object whose ``claim_block_grads(weights)`` may take the
    fp32 weight gradients of a block backward (the sharded optimizer); held by
    weak reference."""
    _SINKS.append(weakref.ref(sink))


def grad_sink_for(weights) -> Optional[tuple]:
    """(fp32 destination [5·H·N·C], fresh) from the first registered sink that
    owns these five weights (q, k, v, g, o), else None."""
    for ref in list(_SINKS):
        sink = ref()
        if sink is None:
            _SINKS.remove(ref)
            continue
        got = sink.claim_block_grads(weights)
        if got is not None:
            return got
    return None
