"""GPU: the block inside its caller.  The reference's module is used in a model
(README.md:1 speaks of a 50M-parameter model); here a small pre-norm residual
stack -- x += attn(x); x += W2 relu(W1 rmsnorm(x))^2, twice -- runs with this
block (bf16, CausalSoftmaxAttention) and with the README's eager block
(README.md:42-64, fp32, plain PyTorch on the GPU) on the same parameters.  The
outputs and the gradients of the input and of every parameter must agree at the
block's own bars (outputs max|a-b|/max|b| <= 3e-2 over two layers, gradient
cosine > 0.999)."""
import math

import pytest
import torch
import torch.nn.functional as F

from gpu_util import DEV, cos, maxrel
from memory_efficient_attn_layer_b200 import CausalSoftmaxAttention, Yarn

pytestmark = pytest.mark.gpu


def _params(L, C, H, N, seed):
    g = torch.Generator().manual_seed(seed)
    P = []
    for _ in range(L):
        b = 0.5 / math.sqrt(C)
        layer = {k: (torch.rand(H * N, C, generator=g) * 2 - 1) * b for k in ("wq", "wk", "wv", "wg")}
        layer["wo"] = (torch.rand(C, H * N, generator=g) * 2 - 1) * 0.5 / math.sqrt(H * N)
        layer["w1"] = (torch.rand(4 * C, C, generator=g) * 2 - 1) / math.sqrt(C)
        layer["w2"] = (torch.rand(C, 4 * C, generator=g) * 2 - 1) / math.sqrt(4 * C)
        P.append(layer)
    return P


def _eager_block(x, p, f1, f2, H, N):
    """README.md:42-64 in fp32: norm, projections, per-head norm + rotary, causal SDPA, gated o_proj."""
    B, T, C = x.shape

    def norm(t):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6)

    def rot(t):
        sw = t.reshape(*t.shape[:-1], N // 2, 2).flip(-1).reshape(t.shape)
        return t * f1[:T].view(1, T, 1, N) + sw * f2[:T].view(1, T, 1, N)

    xn = norm(x)
    q = rot(norm((xn @ p["wq"].t()).view(B, T, H, N)))
    k = rot(norm((xn @ p["wk"].t()).view(B, T, H, N)))
    v = (xn @ p["wv"].t()).view(B, T, H, N)
    g = xn @ p["wg"].t()
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
    o = o.transpose(1, 2).reshape(B, T, H * N)
    return (o * torch.sigmoid(g)) @ p["wo"].t()


def _mlp(h, p):
    return F.linear(F.relu(F.linear(F.rms_norm(h, (h.shape[-1],), eps=1e-6), p["w1"])).square(), p["w2"])


@pytest.mark.parametrize("B,T,C,H,N", [(2, 256, 256, 4, 64), (1, 384, 256, 2, 128)])
def test_residual_stack_matches_eager_fp32(B, T, C, H, N):
    L = 2
    P = _params(L, C, H, N, seed=77)
    gx = torch.Generator().manual_seed(78)
    x0 = torch.randn(B, T, C, generator=gx)
    dy = torch.randn(B, T, C, generator=gx)
    yarn = Yarn(N, T, device=DEV)
    f1, f2 = yarn.factor1.float(), yarn.factor2.float()

    # reference: fp32 eager stack
    Pr = [{k: v.to(DEV).requires_grad_(True) for k, v in layer.items()} for layer in P]
    xr = x0.to(DEV).requires_grad_(True)
    h = xr
    for p in Pr:
        h = h + _eager_block(h, p, f1, f2, H, N)
        h = h + _mlp(h, p)
    h.backward(dy.to(DEV))

    # this build: bf16 stack with the block as CausalSoftmaxAttention modules
    blocks, mlps = [], []
    for p in P:
        m = CausalSoftmaxAttention(C, H, N).to(device=DEV, dtype=torch.bfloat16)
        with torch.no_grad():
            for name, key in (("q_proj", "wq"), ("k_proj", "wk"), ("v_proj", "wv"), ("g_proj", "wg"), ("o_proj", "wo")):
                getattr(m, name).weight.copy_(p[key])
        blocks.append(m)
        mlps.append({k: p[k].to(DEV, torch.bfloat16).requires_grad_(True) for k in ("w1", "w2")})
    xb = x0.to(DEV, torch.bfloat16).requires_grad_(True)
    h2 = xb
    for m, p in zip(blocks, mlps):
        h2 = h2 + m(h2, yarn)
        h2 = h2 + _mlp(h2, p)
    h2.backward(dy.to(DEV, torch.bfloat16))
    torch.cuda.synchronize()

    assert maxrel(h2.detach().float(), h.detach()) <= 3e-2
    assert cos(xb.grad.float(), xr.grad) > 0.999
    for l, (m, pb, pr) in enumerate(zip(blocks, mlps, Pr)):
        for name, key in (("q_proj", "wq"), ("k_proj", "wk"), ("v_proj", "wv"), ("g_proj", "wg"), ("o_proj", "wo")):
            c = cos(getattr(m, name).weight.grad.float(), pr[key].grad)
            assert c > 0.999, (l, key, c)
        for key in ("w1", "w2"):
            c = cos(pb[key].grad.float(), pr[key].grad)
            assert c > 0.999, (l, key, c)
