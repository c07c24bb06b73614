"""Host side of the data-parallel path on CPU: two gloo ranks exchange the
weight gradients through allreduce_grads (coalesced fp32 bucket, mean), the
call the GPU bench makes over NCCL after every backward."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from memory_efficient_attn_layer_b200.dp import active_exchange, allreduce_grads, overlap_grad_allreduce, reduce_weight_grads


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads_for(rank):
    g = torch.Generator().manual_seed(100 + rank)
    shapes = [(64, 32), (64, 32), (64, 32), (64, 32), (32, 64)]
    out = []
    for i, sh in enumerate(shapes):
        p = torch.zeros(sh, dtype=torch.bfloat16 if i < 4 else torch.float32, requires_grad=True)
        p.grad = torch.randn(sh, generator=g).to(p.dtype)
        out.append(p)
    out.append(torch.zeros(3, requires_grad=True))  # no gradient: skipped
    return out


def _worker(rank, world, port, average, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        params = _grads_for(rank)
        allreduce_grads(params, average=average)
        # numpy arrays travel by value: a torch tensor would be fetched from this process after it exits
        q.put((rank, [p.grad.float().numpy() if p.grad is not None else None for p in params]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("average", [True, False])
def test_allreduce_grads_two_ranks(average):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, average, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {r: [None if a is None else torch.from_numpy(a) for a in v]
               for r, v in (q.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = [_grads_for(r) for r in range(world)]
    for i in range(5):
        want = sum(ref[r][i].grad.float() for r in range(world))
        if average:
            want = want / world
        want = want.to(ref[0][i].grad.dtype).float()  # written back in the parameter's dtype
        for r in range(world):
            assert torch.equal(results[r][i], want), (i, r)
    assert results[0][5] is None and results[1][5] is None


def _reduce_worker(rank, world, port, average, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        buf = torch.randn(5 * 12, generator=torch.Generator().manual_seed(7 + rank))
        marks = []
        # the second collective may only start after the callback (the overlapped
        # path's wait on the q/k/v/g readiness event)
        reduce_weight_grads(buf, 4 * 12, average=average, before_qkvg=lambda: marks.append("qkvg"))
        with overlap_grad_allreduce(average=average) as ex:
            tagged = active_exchange() is ex
        q.put((rank, buf.numpy(), marks, tagged))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("average", [True, False])
def test_reduce_weight_grads_two_ranks(average):
    """The overlapped exchange's collectives: o_proj part, callback, q/k/v/g part,
    sum or mean over the group; forwards inside the context get tagged."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reduce_worker, args=(r, world, port, average, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {r: [torch.from_numpy(b), *rest] for r, b, *rest in (q.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = sum(torch.randn(60, generator=torch.Generator().manual_seed(7 + r)) for r in range(world))
    if average:
        want = want / world
    for r in range(world):
        buf, marks, tagged = results[r]
        assert torch.allclose(buf, want, rtol=0, atol=1e-6)
        assert marks == ["qkvg"] and tagged


def test_no_exchange_outside_context_or_without_group():
    assert active_exchange() is None
    with overlap_grad_allreduce():
        assert active_exchange() is None  # no process group: nothing to exchange


def test_bench_resolves_the_exchange_wait_instrument():
    """bench.py --gpus N (N > 1) imports the exchange-wait instrument by name from
    the fused_attn module (the package re-exports a function of the same name)."""
    import ast
    import os

    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")).read()
    names = [(n.module, a.name) for n in ast.walk(ast.parse(src)) if isinstance(n, ast.ImportFrom) for a in n.names]
    assert ("memory_efficient_attn_layer_b200.fused_attn", "record_exchange_waits") in names
    from memory_efficient_attn_layer_b200.fused_attn import record_exchange_waits

    assert record_exchange_waits(True) is None and record_exchange_waits(False) == []
