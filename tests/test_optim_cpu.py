"""CPU: the sharded AdamW step's oracle pinned against torch.optim.AdamW, the
flat shard layout, its two-rank reduce-scatter / all-gather over gloo, and the
argument checks of mea_adamw_step (which reject before any GPU work)."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from memory_efficient_attn_layer_b200 import _lib
from memory_efficient_attn_layer_b200.optim import FlatShards
from oracle.adamw import adamw_step, to_bf16

HYPER = [
    dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-2),
    dict(lr=3e-4, beta1=0.8, beta2=0.95, eps=1e-6, weight_decay=0.0),
    dict(lr=1e-2, beta1=0.0, beta2=0.5, eps=1e-3, weight_decay=0.1),
]


@pytest.mark.parametrize("hp", HYPER)
def test_oracle_matches_torch_adamw(hp):
    g = torch.Generator().manual_seed(3)
    w0 = torch.randn(4099, generator=g)
    p = torch.nn.Parameter(w0.clone())
    opt = torch.optim.AdamW([p], lr=hp["lr"], betas=(hp["beta1"], hp["beta2"]), eps=hp["eps"],
                            weight_decay=hp["weight_decay"], foreach=False)
    master = w0.numpy().copy()
    m = np.zeros_like(master)
    v = np.zeros_like(master)
    gmax = 0.0
    for step in range(1, 7):
        grad = torch.randn(4099, generator=g) * (10.0 ** (step % 3 - 1))
        gmax = max(gmax, float(grad.abs().max()))
        p.grad = grad.clone()
        opt.step()
        adamw_step(master, m, v, grad.numpy(), step=step, **hp)
        np.testing.assert_allclose(master, p.detach().numpy(), rtol=2e-6, atol=1e-7)
        st = opt.state[p]
        # torch's vectorised lerp / addcmul fuse multiply-adds, numpy rounds each
        # operation: a few ulp of the largest gradient seen, carried across steps
        np.testing.assert_allclose(m, st["exp_avg"].numpy(), rtol=1e-5, atol=1e-6 * gmax)
        np.testing.assert_allclose(v, st["exp_avg_sq"].numpy(), rtol=1e-5, atol=1e-6 * gmax * gmax)


def test_oracle_grad_scale_is_a_gradient_multiplier():
    g = np.random.default_rng(0).standard_normal(64).astype(np.float32)
    a = [np.ones(64, np.float32), np.zeros(64, np.float32), np.zeros(64, np.float32)]
    b = [x.copy() for x in a]
    adamw_step(*a, g, step=1, grad_scale=0.5, **HYPER[0])
    adamw_step(*b, g * np.float32(0.5), step=1, **HYPER[0])
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_to_bf16_matches_torch():
    x = torch.randn(100000, generator=torch.Generator().manual_seed(1)) * 37.0
    want = x.to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(to_bf16(x.numpy()), want)


def _params(seed, shapes, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return [torch.nn.Parameter(torch.randn(s, generator=g).to(dtype)) for s in shapes]


def test_flat_layout_views_and_alignment():
    shapes = [(3, 5), (64, 32), (7,), (32, 64)]
    ps = _params(0, shapes)
    before = [p.detach().clone() for p in ps]
    lay = FlatShards(ps)
    assert lay.world == 1 and lay.total % 8 == 0 and lay.shard == lay.total
    for p, o, b in zip(ps, lay.offsets, before):
        assert o % 8 == 0
        assert p.untyped_storage().data_ptr() == lay.flat.untyped_storage().data_ptr()
        assert torch.equal(p.detach(), b)
    lay.flat.zero_()
    assert all(float(p.detach().abs().sum()) == 0 for p in ps)


def test_flat_layout_finds_blocks():
    ps = _params(1, [(64, 32)] * 4 + [(32, 64)] + [(5,)])
    lay = FlatShards(ps)
    assert lay.block_region(ps[:5]) == lay.offsets[0]
    assert lay.block_region([ps[1], ps[0], *ps[2:5]]) is None      # wrong order
    assert lay.block_region(ps[1:6]) is None                       # not five equal blocks
    other = _params(2, [(64, 32)] * 4 + [(32, 64)])
    assert lay.block_region(other) is None                         # not in the flat buffer


def test_add_param_grads_accumulates():
    ps = _params(3, [(4, 4), (3,)])
    lay = FlatShards(ps)
    ps[0].grad = torch.ones(4, 4, dtype=torch.bfloat16)
    lay.add_param_grads()
    lay.add_param_grads()
    assert torch.equal(lay.grad_view(0), torch.full((4, 4), 2.0))
    assert float(lay.grad_view(1).abs().sum()) == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SHAPES = [(48, 40), (48, 40), (13,), (40, 48)]
HP = HYPER[0]


def _rank_grads(rank):
    g = torch.Generator().manual_seed(50 + rank)
    return [torch.randn(s, generator=g).to(torch.bfloat16) for s in SHAPES]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ps = _params(7 + rank, SHAPES)  # different on each rank: the layout broadcasts rank 0's
        lay = FlatShards(ps)
        for p, gr in zip(ps, _rank_grads(rank)):
            p.grad = gr
        lay.add_param_grads()
        gshard = torch.empty(lay.shard)
        lay.reduce_scatter(gshard)
        lo = lay.lo
        master = lay.flat[lo:lo + lay.shard].float().numpy().copy()
        m = np.zeros_like(master)
        v = np.zeros_like(master)
        new = adamw_step(master, m, v, gshard.numpy(), step=1, grad_scale=1.0 / world, **HP)
        lay.all_gather(torch.from_numpy(new).to(torch.bfloat16))
        # numpy arrays travel by value: a torch tensor would be fetched from this process after it exits
        q.put((rank, lay.flat.float().numpy(), [p.detach().float().numpy() for p in ps]))
    finally:
        dist.destroy_process_group()


def test_two_rank_reduce_scatter_step_all_gather():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, flat, ps = q.get(timeout=120)
        got[r] = (torch.from_numpy(flat), [torch.from_numpy(p) for p in ps])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # One process, no sharding: rank 0's weights, the mean gradient, one step.
    ps0 = _params(7, SHAPES)
    lay = FlatShards(ps0)
    for i in range(len(SHAPES)):
        lay.grad_view(i).copy_(sum(_rank_grads(r)[i].float() for r in range(world)))
    master = lay.flat.float().numpy().copy()
    new = adamw_step(master, np.zeros_like(master), np.zeros_like(master), lay.grad32.numpy(), step=1,
                     grad_scale=1.0 / world, **HP)
    want = torch.from_numpy(new)
    for r in range(world):
        flat, ps = got[r]
        assert torch.equal(flat[:lay.numel], want[:lay.numel]), r
        for i, p in enumerate(ps):
            o = lay.offsets[i]
            assert torch.equal(p.flatten(), want[o:o + p.numel()]), (r, i)


# ---- argument checks of the C entry point (no GPU work is reached) ----------------

def _call(L, n, ptrs, step=1, betas=(0.9, 0.999), lr=1e-3, eps=1e-8, wd=0.0):
    return L.mea_adamw_step(n, *ptrs, lr, betas[0], betas[1], eps, wd, 1.0, step, None)


def test_adamw_entry_rejects_bad_arguments():
    L = _lib.lib()
    ok = [ctypes.c_void_p(256)] * 4 + [ctypes.c_void_p(512)]
    assert _call(L, 0, [None] * 5) == 0
    assert _call(L, -1, ok) == 1
    assert _call(L, 4, [None] + ok[1:]) == 1
    assert _call(L, 4, ok, step=0) == 1 and b"step" in L.mea_last_error_string()
    assert _call(L, 4, ok, betas=(1.0, 0.999)) == 1 and b"betas" in L.mea_last_error_string()
    assert _call(L, 4, ok, lr=-1.0) == 1
    assert _call(L, 4, [ctypes.c_void_p(260)] + ok[1:]) == 3
    assert _call(L, 4, ok[:4] + [ctypes.c_void_p(514)]) == 3
