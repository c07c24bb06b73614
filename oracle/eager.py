"""CPU oracle for the gated causal attention block -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it.  The CUDA path in ``memory_efficient_attn_layer_b200`` never calls it.

It restates, in plain fp32/fp64 PyTorch on the CPU, the eager block that the
reference declares equivalent to ``fused_attn`` (README.md:3 and the
commented-out code at README.md:42-64), with the numerics of the reference
kernels where the README leaves them open:

* ``norm``  -- parameter-free RMSNorm, mean over the last dim, ``rsqrt(var+eps)``
  with eps = 1e-6 (fast_triton_attn.py:29-32, default eps at :681).
* per-head q/k RMSNorm over the head dim N (fast_triton_attn.py:102-106).
* rotary -- ``x * f1 + swap_even_odd(x) * f2`` where ``swap_even_odd`` flips the
  pair (2i, 2i+1) (fast_triton_attn.py:132-141 and :497-498).
* causal softmax attention with scale 1/sqrt(N) (fast_triton_attn.py:426, :438).
* gate ``o * sigmoid(g)`` before o_proj (fast_triton_attn.py:123, :171;
  README.md:64).

Gradients come from autograd on this forward, so they are exact for any
factor table (the reference's backward at fast_triton_attn.py:603-639 is exact
only for orthogonal tables).

Parity of this oracle is pinned against outputs of the reference's own
``FusedAttentionFunction`` run in the build container (fixtures under
``tests/golden/`` and the script that made them, ``tests/golden/make_golden.py``).
The rotary tables themselves (the reference's ``yarn`` object) are not part of
the reference, so the tables are an input on both sides.
"""
from __future__ import annotations

import math
from typing import Dict, Sequence

import torch


def rms_norm(x: torch.Tensor, eps: float) -> torch.Tensor:
    """Parameter-free RMSNorm over the last dim (fast_triton_attn.py:29-32)."""
    return x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)


def swap_even_odd(x: torch.Tensor) -> torch.Tensor:
    """Swap elements 2i and 2i+1 of the last dim (fast_triton_attn.py:497-498)."""
    return x.reshape(*x.shape[:-1], x.shape[-1] // 2, 2).flip(-1).reshape(x.shape)


def rotary(x: torch.Tensor, f1: torch.Tensor, f2: torch.Tensor) -> torch.Tensor:
    """Interleaved rotary ``x*f1 + swap(x)*f2`` (fast_triton_attn.py:132-141)."""
    return x * f1 + swap_even_odd(x) * f2


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """softmax(q k^T * scale, causal) v for [B, H, T, N] tensors (fast_triton_attn.py:438)."""
    T = q.shape[-2]
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    mask = torch.ones(T, T, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v)


def block_forward(x, wq, wk, wv, wg, wo, factor1, factor2, H: int, N: int, eps: float = 1e-6):
    """The eager block of README.md:42-64.

    x: [B, T, C]; wq/wk/wv/wg: [H*N, C]; wo: [C, H*N]; factor1/2: [T_max >= T, N].
    Returns y: [B, T, C].
    """
    B, T, C = x.shape
    xn = rms_norm(x, eps)                                   # README:43
    q = (xn @ wq.t()).view(B, T, H, N)                      # README:45
    k = (xn @ wk.t()).view(B, T, H, N)                      # README:46
    v = (xn @ wv.t()).view(B, T, H, N)                      # README:47
    g = xn @ wg.t()                                         # README:48
    f1 = factor1[:T].view(1, T, 1, N)
    f2 = factor2[:T].view(1, T, 1, N)
    q = rotary(rms_norm(q, eps), f1, f2)                    # README:50
    k = rotary(rms_norm(k, eps), f1, f2)
    o = causal_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                         1.0 / math.sqrt(N))                # README:56-62
    o = o.transpose(1, 2).reshape(B, T, H * N)
    return (o * torch.sigmoid(g)) @ wo.t()                  # README:64


GRAD_NAMES = ("dx", "dwq", "dwk", "dwv", "dwg", "dwo", "df1", "df2")


def block_fwd_bwd(inputs: Dict[str, torch.Tensor], H: int, N: int, eps: float = 1e-6,
                  dtype: torch.dtype = torch.float32,
                  factor_grads: bool = True) -> Dict[str, torch.Tensor]:
    """Forward + backward of the eager block on the CPU in ``dtype``.

    ``inputs`` holds x, wq, wk, wv, wg, wo, f1, f2 and dy (upstream gradient).
    Returns y and the gradients named in ``GRAD_NAMES`` (df1/df2 only when
    ``factor_grads``), all in ``dtype``.  The gradient tuple matches the order
    that the reference backward returns (fast_triton_attn.py:671-675).
    """
    names = ("x", "wq", "wk", "wv", "wg", "wo", "f1", "f2")
    leaves = []
    for n in names:
        t = inputs[n].detach().to("cpu", dtype).clone()
        t.requires_grad_(n not in ("f1", "f2") or factor_grads)
        leaves.append(t)
    y = block_forward(*leaves, H=H, N=N, eps=eps)
    y.backward(inputs["dy"].detach().to("cpu", dtype))
    out = {"y": y.detach()}
    for gname, leaf in zip(GRAD_NAMES, leaves):
        if leaf.requires_grad:
            out[gname] = leaf.grad.detach()
    return out


def yarn_tables(N: int, T_max: int, base: float = 10000.0, mscale: float = 1.0):
    """Interleaved rotary tables used as the stand-in for the reference's ``yarn``.

    factor1[t, 2i] = factor1[t, 2i+1] = mscale*cos(t*theta_i) and
    factor2[t, 2i] = -mscale*sin(t*theta_i), factor2[t, 2i+1] = +mscale*sin(t*theta_i),
    theta_i = base^(-2i/N).  With these, ``rotary`` is the standard pairwise
    rotation (times ``mscale``).  The reference reads ``yarn.factor1/2``
    (fast_triton_attn.py:692-693) but does not define them.
    """
    inv = base ** (-torch.arange(0, N, 2, dtype=torch.float64) / N)
    ang = torch.arange(T_max, dtype=torch.float64)[:, None] * inv[None, :]
    c, s = torch.cos(ang) * mscale, torch.sin(ang) * mscale
    f1 = torch.stack([c, c], dim=-1).reshape(T_max, N)
    f2 = torch.stack([-s, s], dim=-1).reshape(T_max, N)
    return f1.float(), f2.float()


def make_inputs(B: int, T: int, C: int, H: int, N: int, seed: int = 0,
                mscale: float = 1.0, T_max: int | None = None,
                round_bf16: bool = True) -> Dict[str, torch.Tensor]:
    """Seeded synthetic inputs with the distributions the baseline configs name.

    x ~ N(0,1); q/k/v/g/o weights ~ U(-0.5/sqrt(C), 0.5/sqrt(C)) (README.md:21-32,
    with o_proj non-zero so gradients flow); dy ~ N(0,1).  All tensors are
    fp32 on the CPU; with ``round_bf16`` they are rounded to bf16-representable
    values so that a bf16 device path and an fp32 CPU path see identical inputs.
    """
    g = torch.Generator().manual_seed(seed)
    HN = H * N
    bound = 0.5 / math.sqrt(C)
    x = torch.randn(B, T, C, generator=g)
    ws = [torch.empty(HN, C).uniform_(-bound, bound, generator=g) for _ in range(4)]
    wo = torch.empty(C, HN).uniform_(-bound, bound, generator=g)
    dy = torch.randn(B, T, C, generator=g)
    f1, f2 = yarn_tables(N, T_max or T, mscale=mscale)
    d = dict(x=x, wq=ws[0], wk=ws[1], wv=ws[2], wg=ws[3], wo=wo, f1=f1, f2=f2, dy=dy)
    if round_bf16:
        d = {k: v.to(torch.bfloat16).float() for k, v in d.items()}
    return d


def max_rel(a: torch.Tensor, b: torch.Tensor) -> float:
    """max|a - b| / max|b|: the output tolerance measure used by the parity tests."""
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def cos_sim(a: torch.Tensor, b: torch.Tensor) -> float:
    """Cosine similarity of two tensors viewed as flat vectors."""
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-300))


def compare(got: Dict[str, torch.Tensor], want: Dict[str, torch.Tensor],
            names: Sequence[str]) -> Dict[str, Dict[str, float]]:
    """max_rel and cos_sim for each named tensor."""
    return {n: {"max_rel": max_rel(got[n], want[n]), "cos": cos_sim(got[n], want[n])}
            for n in names}
