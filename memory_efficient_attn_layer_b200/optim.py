"""Sharded AdamW for the block's weights: reduce-scatter, one fused update
kernel, all-gather.

Data-parallel ranks hold the same weights and their own gradients.  Instead
of all-reducing every gradient and then updating every weight on every rank,
``ShardedAdamW`` cuts the flattened weights into ``world`` equal shards:

1. the fp32 gradients are reduce-scattered (sum), so rank r receives the sum
   for shard r only;
2. ``mea_adamw_step`` (one kernel, one HBM pass) updates shard r's fp32 master
   weights and both moments and writes the new bf16 weights of the shard;
3. the bf16 shards are all-gathered into the flat buffer that every
   parameter's storage is a view of.

Each rank keeps 12 bytes of optimizer state per weight for 1/world of the
weights, and moves (4 + 2)·P·(world-1)/world bytes per step where an fp32
all-reduce moves 8·P·(world-1)/world.

Gradients of a ``FusedAttentionFunction`` whose five weights are consecutive
views of the flat buffer in the order q, k, v, g, o (the order
``CausalSoftmaxAttention`` creates its projections in, README.md:21-32) are
written by the block's backward straight into the optimizer's fp32 gradient
buffer: no bf16 rounding of the weight gradients and no cast kernel.  Those
weights' ``.grad`` stay None.  Any other ``.grad`` of the managed parameters
is added in at ``step()``.  ``zero_grad()`` clears both.
"""
from __future__ import annotations

from typing import Iterable, Optional

import torch
import torch.distributed as dist

from . import _lib
from . import dp as _dp

_ALIGN = 8  # elements: every parameter starts 16-byte aligned in bf16, 32-byte in fp32


def _round_up(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def _group_size_rank(group) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


class FlatShards:
    """Flat, rank-sharded layout of a list of same-dtype tensors; no arithmetic.

    Parameter i occupies ``flat[offsets[i] : offsets[i] + numel]``, each offset
    a multiple of 8 elements; the total is padded to a multiple of 8·world so
    that rank r's shard ``[r·S, (r+1)·S)`` is 16-byte aligned.  Every tensor's
    ``.data`` becomes a view of ``flat``.  ``grad32`` is the fp32 gradient
    buffer with the same layout.  With ``broadcast`` the group's first rank's
    values are copied to every rank (ranks must start from identical weights).
    """

    def __init__(self, params: list, group=None, broadcast: bool = True):
        if not params:
            raise ValueError("no parameters to shard")
        dtype, device = params[0].dtype, params[0].device
        seen = set()
        for p in params:
            if p.dtype != dtype or p.device != device:
                raise TypeError("all parameters must share one dtype and device")
            if id(p) in seen:
                raise ValueError("a parameter appears twice")
            seen.add(id(p))
        self.group = group
        self.world, self.rank = _group_size_rank(group)
        self.params = params
        self.offsets, off = [], 0
        for p in params:
            off = _round_up(off, _ALIGN)
            self.offsets.append(off)
            off += p.numel()
        self.numel = off
        self.total = _round_up(max(off, 1), _ALIGN * self.world)
        self.shard = self.total // self.world
        self.flat = torch.zeros(self.total, dtype=dtype, device=device)
        with torch.no_grad():
            for p, o in zip(params, self.offsets):
                self.flat[o:o + p.numel()].copy_(p.detach().reshape(-1))
            if broadcast and self.world > 1:
                dist.broadcast(self.flat, src=dist.get_global_rank(group, 0) if group is not None else 0,
                               group=group)
            for p, o in zip(params, self.offsets):
                p.data = self.flat[o:o + p.numel()].view(p.shape)
        self.grad32 = torch.zeros(self.total, dtype=torch.float32, device=device)

    @property
    def lo(self) -> int:
        return self.rank * self.shard

    def grad_view(self, i: int) -> torch.Tensor:
        o, p = self.offsets[i], self.params[i]
        return self.grad32[o:o + p.numel()].view(p.shape)

    def add_param_grads(self) -> None:
        """grad32 += p.grad for every parameter that has one."""
        for i, p in enumerate(self.params):
            if p.grad is not None:
                self.grad_view(i).add_(p.grad)

    def reduce_scatter(self, out: torch.Tensor) -> None:
        """out (fp32 [S]) <- sum over the group of grad32[r·S : (r+1)·S]."""
        if self.world == 1:
            if out.data_ptr() != self.grad32.data_ptr():
                out.copy_(self.grad32)
            return
        dist.reduce_scatter_tensor(out, self.grad32, group=self.group)

    def all_gather(self, shard_values: torch.Tensor) -> None:
        """flat <- every rank's shard (shard_values: [S], flat's dtype)."""
        if self.world == 1:
            if shard_values.data_ptr() != self.flat.data_ptr():
                self.flat.copy_(shard_values)
            return
        dist.all_gather_into_tensor(self.flat, shard_values, group=self.group)

    def block_region(self, weights) -> Optional[int]:
        """Offset in grad32 of five tensors that are consecutive views of flat
        (q, k, v, g, o, equal sizes, contiguous), else None."""
        if len(weights) != 5:
            return None
        base = self.flat.untyped_storage().data_ptr()
        n = weights[0].numel()
        first = weights[0].storage_offset()
        for j, w in enumerate(weights):
            if (w.untyped_storage().data_ptr() != base or not w.is_contiguous() or w.numel() != n
                    or w.storage_offset() != first + j * n):
                return None
        if first % _ALIGN or first not in self.offsets:
            return None
        return first


class ShardedAdamW(torch.optim.Optimizer):
    """AdamW (torch.optim.AdamW's update, decoupled weight decay) over bf16
    parameters, with fp32 master weights and moments sharded across the
    data-parallel ``group`` (see the module docstring).  One parameter group.

    ``average``: the gradient is the mean over ranks (each rank's loss a mean
    over its own batch shard); otherwise the sum.  ``fused_grads``: accept the
    block backward's fp32 weight gradients directly (their ``.grad`` stays
    None).  The weights must start identical on every rank; the first rank's
    are broadcast at construction.

    Every ``step()`` updates every managed weight: a weight that received no
    gradient since ``zero_grad()`` is stepped with a zero gradient (its moments
    decay and weight decay applies), where torch.optim.AdamW would skip it.
    Under data parallelism every rank must call ``step()`` the same number of
    times, as for any collective."""

    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-3, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2, group=None, average: bool = True,
                 fused_grads: bool = True):
        params = list(params)
        if not lr >= 0.0:
            raise ValueError(f"invalid learning rate {lr}")
        if not eps >= 0.0:
            raise ValueError(f"invalid eps {eps}")
        if not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"invalid betas {betas}")
        if not weight_decay >= 0.0:
            raise ValueError(f"invalid weight_decay {weight_decay}")
        for p in params:
            if p.dtype != torch.bfloat16:
                raise TypeError(f"ShardedAdamW updates bf16 parameters; got {p.dtype}")
        if not params:
            raise ValueError("ShardedAdamW got an empty parameter list")
        _lib.require_device(params[0].device)
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))
        self.layout = FlatShards(params, group)
        self.average = average
        self.fused_grads = fused_grads
        L = self.layout
        lo, S = L.lo, L.shard
        self.master = L.flat[lo:lo + S].float()
        self.exp_avg = torch.zeros(S, dtype=torch.float32, device=L.flat.device)
        self.exp_avg_sq = torch.zeros(S, dtype=torch.float32, device=L.flat.device)
        single = L.world == 1
        self.grad_shard = L.grad32 if single else torch.empty(S, dtype=torch.float32, device=L.flat.device)
        self.param_shard = L.flat if single else torch.empty(S, dtype=torch.bfloat16, device=L.flat.device)
        self.steps = 0
        self._written = set()
        _dp.register_grad_sink(self)

    # -- gradients from the block's backward ------------------------------------------
    def claim_block_grads(self, weights) -> Optional[tuple[torch.Tensor, bool]]:
        """(fp32 view of the five weights' gradient region, fresh) when the
        weights are a block of this optimizer; ``fresh`` is False when that
        region already holds a gradient since the last ``zero_grad()`` (the
        caller then adds into it instead of overwriting)."""
        if not self.fused_grads:
            return None
        off = self.layout.block_region(weights)
        if off is None:
            return None
        fresh = off not in self._written
        self._written.add(off)
        return self.layout.grad32[off:off + 5 * weights[0].numel()], fresh

    def zero_grad(self, set_to_none: bool = True) -> None:
        super().zero_grad(set_to_none)
        self.layout.grad32.zero_()
        self._written.clear()

    # -- the step -----------------------------------------------------------------------
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        L = self.layout
        g = self.param_groups[0]
        self.steps += 1
        L.add_param_grads()
        L.reduce_scatter(self.grad_shard)
        scale = 1.0 / L.world if self.average else 1.0
        lib = _lib.lib()
        dev = L.flat.device
        _lib.check(lib.mea_adamw_step(
            L.shard, _lib.ptr(self.master), _lib.ptr(self.exp_avg), _lib.ptr(self.exp_avg_sq),
            _lib.ptr(self.grad_shard), _lib.ptr(self.param_shard), float(g["lr"]), float(g["betas"][0]),
            float(g["betas"][1]), float(g["eps"]), float(g["weight_decay"]), scale, self.steps,
            _lib.stream_ptr(dev)))
        L.all_gather(self.param_shard)
        return loss

    # -- checkpoints (this rank's shard) ---------------------------------------------
    def state_dict(self) -> dict:
        L = self.layout
        return {"steps": self.steps, "world": L.world, "rank": L.rank, "total": L.total,
                "master": self.master.clone(), "exp_avg": self.exp_avg.clone(),
                "exp_avg_sq": self.exp_avg_sq.clone(),
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def load_state_dict(self, state: dict) -> None:
        L = self.layout
        if (state["world"], state["rank"], state["total"]) != (L.world, L.rank, L.total):
            raise ValueError("state was saved for another shard layout "
                             f"(world {state['world']}, rank {state['rank']}, total {state['total']})")
        with torch.no_grad():
            self.master.copy_(state["master"])
            self.exp_avg.copy_(state["exp_avg"])
            self.exp_avg_sq.copy_(state["exp_avg_sq"])
            lo = L.lo
            L.flat[lo:lo + L.shard].copy_(self.master.to(torch.bfloat16))
        self.steps = int(state["steps"])
        for g, saved in zip(self.param_groups, state["param_groups"]):
            g.update(saved)
        if L.world > 1:
            L.all_gather(L.flat[L.lo:L.lo + L.shard].clone())
