"""GPU: the sharded AdamW step.

* mea_adamw_step against the CPU oracle: fp32 master weights and moments
  within a few ulp (the kernel fuses multiply-adds, the oracle rounds every
  operation: rtol 1e-5); the bf16 weights are the kernel's own fp32 master
  rounded to nearest even, bit for bit.
* ShardedAdamW on the block: the backward's fp32 weight gradients land in the
  optimizer's buffer (cosine > 0.9999 against the bf16 gradients of the plain
  backward; two backwards accumulate), ``.grad`` stays None, and one step
  equals the oracle applied to that buffer.
* Two GPUs over NCCL (reduce-scatter, step, all-gather) equal one GPU on the
  full batch (skipped with fewer than two GPUs).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from gpu_util import DEV, P, call, cos, stream
from oracle.adamw import adamw_step, to_bf16

pytestmark = pytest.mark.gpu
HP = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-2)


@pytest.mark.parametrize("n", [1, 7, 4099, (1 << 20) + 5])
def test_adamw_kernel_matches_oracle(n):
    g = torch.Generator().manual_seed(n)
    master = torch.randn(n, generator=g)
    dm = master.to(DEV)
    dexp = torch.zeros(n, device=DEV)
    dsq = torch.zeros(n, device=DEV)
    p = torch.empty(n, dtype=torch.bfloat16, device=DEV)
    om, oexp, osq = master.numpy().copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    gmax = 0.0
    for step in range(1, 4):
        grad = torch.randn(n, generator=g) * (10.0 ** (step - 2))
        gmax = max(gmax, float(grad.abs().max()))
        dgrad = grad.to(DEV)
        call("mea_adamw_step", n, P(dm), P(dexp), P(dsq), P(dgrad), P(p), HP["lr"], HP["beta1"], HP["beta2"],
             HP["eps"], HP["weight_decay"], 0.5, step, stream())
        adamw_step(om, oexp, osq, grad.numpy(), step=step, grad_scale=0.5, **HP)
        got = dm.cpu().numpy()
        np.testing.assert_allclose(got, om, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(dexp.cpu().numpy(), oexp, rtol=1e-5, atol=1e-6 * gmax)
        np.testing.assert_allclose(dsq.cpu().numpy(), osq, rtol=1e-5, atol=1e-6 * gmax * gmax)
        np.testing.assert_array_equal(p.float().cpu().numpy(), to_bf16(got))


def test_adamw_kernel_without_bf16_copy():
    n = 1000
    dm = torch.ones(n, device=DEV)
    z = [torch.zeros(n, device=DEV) for _ in range(2)]
    grad = torch.full((n,), 2.0, device=DEV)
    call("mea_adamw_step", n, P(dm), P(z[0]), P(z[1]), P(grad), None, 0.1, 0.9, 0.999, 0.0, 0.0, 1.0, 1, stream())
    # step 1 with eps = 0: m_hat / sqrt(v_hat) = sign(g) = 1, so w = 1 - lr
    assert torch.allclose(dm, torch.full_like(dm, 0.9), rtol=0, atol=1e-6)


def _module(dev=DEV, C=256, H=4, N=64, seed=5):
    from memory_efficient_attn_layer_b200 import CausalSoftmaxAttention, Yarn

    torch.manual_seed(seed)  # the projections are initialised on the CPU generator
    mod = CausalSoftmaxAttention(C, H, N)
    with torch.no_grad():  # o_proj non-zero so every gradient flows
        b = 0.5 / C ** 0.5
        mod.o_proj.weight.copy_(torch.empty(C, H * N).uniform_(-b, b, generator=torch.Generator().manual_seed(seed)))
    return mod.to(device=dev, dtype=torch.bfloat16), Yarn(N, 512, device=dev)


def _batch(B, T, C, dev=DEV, seed=9):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, C, generator=g).to(dev, torch.bfloat16)
    dy = torch.randn(B, T, C, generator=g).to(dev, torch.bfloat16)
    return x, dy


def _weights(mod):
    return [mod.q_proj.weight, mod.k_proj.weight, mod.v_proj.weight, mod.g_proj.weight, mod.o_proj.weight]


def test_sharded_adamw_takes_the_block_gradients_and_steps():
    from memory_efficient_attn_layer_b200.optim import ShardedAdamW

    mod, yarn = _module()
    x, dy = _batch(2, 256, 256)
    # Plain backward first: the bf16 gradients to compare against.
    mod(x, yarn).backward(dy)
    want = [w.grad.float().flatten() for w in _weights(mod)]
    for w in _weights(mod):
        w.grad = None
    opt = ShardedAdamW(_weights(mod), **{k: v for k, v in HP.items() if k not in ("beta1", "beta2")},
                       betas=(HP["beta1"], HP["beta2"]))
    mod(x, yarn).backward(dy)
    assert all(w.grad is None for w in _weights(mod))
    lay = opt.layout
    got = [lay.grad_view(i).flatten() for i in range(5)]
    for i in range(5):
        assert cos(got[i], want[i]) > 0.9999, i
    once = lay.grad32.clone()
    mod(x, yarn).backward(dy)  # no zero_grad: accumulates
    assert cos(lay.grad32, 2 * once) > 0.99999
    # One step against the oracle on the buffer's contents.
    g32 = lay.grad32.cpu().numpy().copy()
    master = lay.flat.float().cpu().numpy().copy()
    want_w = adamw_step(master, np.zeros_like(master), np.zeros_like(master), g32, step=1, **HP)
    opt.step()
    torch.cuda.synchronize()
    got_master = opt.master.cpu().numpy()
    np.testing.assert_allclose(got_master, master, rtol=1e-5, atol=1e-6)
    new = lay.flat.float().cpu().numpy()
    assert (new != want_w).mean() < 1e-3  # bf16 ties of a few-ulp master difference
    np.testing.assert_array_equal(new, to_bf16(got_master))
    for i, w in enumerate(_weights(mod)):
        o = lay.offsets[i]
        assert torch.equal(w.detach().flatten().float().cpu(), torch.from_numpy(new[o:o + w.numel()]))
    opt.zero_grad()
    assert float(lay.grad32.abs().sum()) == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _train(dev, lo, hi, steps):
    from memory_efficient_attn_layer_b200.optim import ShardedAdamW

    mod, yarn = _module(dev)
    x, dy = _batch(4, 256, 256, dev)
    x, dy = x[lo:hi].contiguous(), dy[lo:hi].contiguous()
    opt = ShardedAdamW(_weights(mod), lr=1e-2, eps=1e-3, weight_decay=0.0, average=False)
    for _ in range(steps):
        opt.zero_grad()
        mod(x, yarn).backward(dy)
        opt.step()
    torch.cuda.synchronize(dev)
    return [w.detach().float().cpu() for w in _weights(mod)]


def _rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        per = 4 // world
        # numpy arrays travel by value: a torch tensor would be fetched from this process after it exits
        q.put((rank, [w.numpy() for w in _train(dev, rank * per, (rank + 1) * per, 3)]))
    finally:
        dist.destroy_process_group()


def test_sharded_adamw_two_ranks_match_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {r: [torch.from_numpy(a) for a in v] for r, v in (q.get(timeout=300) for _ in range(world))}
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    start = [w.detach().float().cpu() for w in _weights(_module()[0])]
    full = _train(DEV, 0, 4, 3)
    for i in range(5):
        assert torch.equal(got[0][i], got[1][i]), i  # the all-gather leaves every rank identical
        c = cos((got[0][i] - start[i]).flatten(), (full[i] - start[i]).flatten())
        assert c > 0.999, (i, c)
