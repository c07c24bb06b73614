"""GPU, 2 ranks: the data-parallel path end to end.  Each rank runs the block
on its half of the batch and the five weight gradients are exchanged over NCCL
(sum), either with allreduce_grads after the backward or overlapped with the
backward (overlap_grad_allreduce); they must equal one GPU's full-batch weight
gradients (cosine > 0.9999; bf16 gradients summed in fp32).  Skipped with fewer
than two GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
SHAPE = dict(B=4, T=256, C=256, H=4, N=64)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from oracle.eager import make_inputs

    return make_inputs(SHAPE["B"], SHAPE["T"], SHAPE["C"], SHAPE["H"], SHAPE["N"], seed=41)


def _weight_grads(inp, dev, lo, hi, exchange=None):
    import contextlib

    from memory_efficient_attn_layer_b200 import FusedAttentionFunction

    leaves = [inp[k].to(device=dev, dtype=torch.bfloat16).contiguous() for k in ("wq", "wk", "wv", "wg", "wo")]
    for w in leaves:
        w.requires_grad_(True)
    x = inp["x"][lo:hi].to(device=dev, dtype=torch.bfloat16).contiguous()
    f1 = inp["f1"].to(device=dev, dtype=torch.bfloat16).contiguous()
    f2 = inp["f2"].to(device=dev, dtype=torch.bfloat16).contiguous()
    with exchange if exchange is not None else contextlib.nullcontext():
        y = FusedAttentionFunction.apply(x, *leaves, f1, f2, SHAPE["H"], SHAPE["N"], 1e-6)
        y.backward(inp["dy"][lo:hi].to(device=dev, dtype=torch.bfloat16))
    return leaves


def _rank(rank, world, port, overlap, q):
    import datetime

    import torch.distributed as dist

    from memory_efficient_attn_layer_b200.dp import allreduce_grads, overlap_grad_allreduce

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        inp = _inputs()
        per = SHAPE["B"] // world
        if overlap:
            leaves = _weight_grads(inp, dev, rank * per, (rank + 1) * per, overlap_grad_allreduce(average=False))
        else:
            leaves = _weight_grads(inp, dev, rank * per, (rank + 1) * per)
            allreduce_grads(leaves, average=False)
        torch.cuda.synchronize(dev)
        # numpy arrays travel by value: a torch tensor would be fetched from this process after it exits
        q.put((rank, [w.grad.float().cpu().numpy() for w in leaves]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("overlap", [False, True])
def test_dp_two_ranks_match_full_batch(overlap):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, overlap, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {r: [torch.from_numpy(a) for a in v] for r, v in (q.get(timeout=300) for _ in range(world))}
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = _weight_grads(_inputs(), torch.device("cuda", 0), 0, SHAPE["B"])
    for i, w in enumerate(full):
        want = w.grad.float().cpu()
        for r in range(world):
            c = torch.nn.functional.cosine_similarity(got[r][i].flatten(), want.flatten(), dim=0).item()
            assert c > 0.9999, (i, r, c)
