"""``CausalSoftmaxAttention`` (README.md:6-68) and the rotary-table object it reads.

The reference's module calls ``fused_attn(x, q_proj, k_proj, v_proj, g_proj,
o_proj, yarn, H, N)`` with a ``yarn`` object that exposes ``factor1``,
``factor2`` ([T_max, N]) and ``rotary()`` (fast_triton_attn.py:692-693,
README.md:50); that object is not part of the reference.  ``Yarn`` here
provides it: interleaved rotary tables with the standard RoPE frequencies and
optional YaRN context extension (NTK-by-parts frequency interpolation and the
attention magnitude scale of Peng et al., 2023, "YaRN: Efficient Context
Window Extension of Large Language Models").
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .fused_attn import fused_attn


def _swap_even_odd(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(*x.shape[:-1], x.shape[-1] // 2, 2).flip(-1).reshape(x.shape)


class Yarn(nn.Module):
    """Interleaved rotary tables ``factor1`` / ``factor2`` of shape [max_seq, head_dim].

    factor1[t, 2i] = factor1[t, 2i+1] = m*cos(t*theta_i);
    factor2[t, 2i] = -m*sin(t*theta_i), factor2[t, 2i+1] = +m*sin(t*theta_i),
    so ``rotary(x) = x*factor1 + swap_even_odd(x)*factor2`` rotates each pair
    (2i, 2i+1) by t*theta_i (fast_triton_attn.py:132-141) and scales by m.

    With ``scale == 1``: theta_i = base^(-2i/N), m = 1.
    With ``scale > 1`` (YaRN, "NTK-by-parts"): pair i keeps theta_i (extrapolation)
    below the correction range, takes theta_i/scale (interpolation) above it, and
    is blended linearly in the pair index inside it.  The range runs from the
    pair index that makes ``beta_fast`` rotations over the original context to
    the one that makes ``beta_slow``, d(r) = N ln(L / (2 pi r)) / (2 ln base),
    rounded outwards (floor / ceil) and clamped to [0, N-1], as in the published
    YaRN reference code; m = 0.1*ln(scale) + 1 unless ``mscale`` is given.
    """

    def __init__(self, head_dim: int, max_seq: int, base: float = 10000.0, scale: float = 1.0,
                 original_max_seq: int | None = None, beta_fast: float = 32.0, beta_slow: float = 1.0,
                 mscale: float | None = None, dtype: torch.dtype = torch.bfloat16, device=None):
        super().__init__()
        if head_dim % 2:
            raise ValueError("head_dim must be even")
        self.head_dim, self.max_seq = head_dim, max_seq
        inv = base ** (-torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
        m = 1.0
        if scale > 1.0:
            orig = original_max_seq or max_seq

            def corr_dim(rotations):  # pair-index coordinate d (in units of N) making `rotations` turns over orig
                return head_dim * math.log(orig / (rotations * 2 * math.pi)) / (2 * math.log(base))

            low = max(math.floor(corr_dim(beta_fast)), 0)
            high = min(math.ceil(corr_dim(beta_slow)), head_dim - 1)
            if low == high:
                high += 0.001
            ramp = ((torch.arange(head_dim // 2, dtype=torch.float64) - low) / (high - low)).clamp(0.0, 1.0)
            inv = inv / scale * ramp + inv * (1.0 - ramp)
            m = 0.1 * math.log(scale) + 1.0
        if mscale is not None:
            m = mscale
        self.inv_freq, self.mscale = inv, m
        ang = torch.arange(max_seq, dtype=torch.float64)[:, None] * inv[None, :]
        c, s = torch.cos(ang) * m, torch.sin(ang) * m
        f1 = torch.stack([c, c], dim=-1).reshape(max_seq, head_dim)
        f2 = torch.stack([-s, s], dim=-1).reshape(max_seq, head_dim)
        self.register_buffer("factor1", f1.to(dtype=dtype, device=device), persistent=False)
        self.register_buffer("factor2", f2.to(dtype=dtype, device=device), persistent=False)

    def rotary(self, x: torch.Tensor) -> torch.Tensor:
        """Apply the rotation to x[..., T, (H,) N] laid out as [B, T, H, N] (README.md:50)."""
        T = x.shape[1]
        shape = [1, T] + [1] * (x.dim() - 3) + [self.head_dim]
        f1 = self.factor1[:T].view(shape).to(x.dtype)
        f2 = self.factor2[:T].view(shape).to(x.dtype)
        return x * f1 + _swap_even_odd(x) * f2


class CausalSoftmaxAttention(nn.Module):
    """The reference block module (README.md:6-68): five bias-free projections,
    q/k/v/g: C -> H*N initialised U(+-0.5/sqrt(C)); o: H*N -> C zero-initialised.
    ``save_o`` (default off) keeps the attention output for the backward
    instead of recomputing it there."""

    def __init__(self, input_dim: int, num_heads: int, head_dim: int, save_o: bool = False):
        super().__init__()
        self.head_dim = head_dim
        self.num_heads = num_heads
        self.save_o = save_o
        N, H, C = head_dim, num_heads, input_dim
        with torch.no_grad():
            bound = 0.5 / (C ** 0.5)
            self.q_proj = nn.Linear(C, H * N, bias=False)
            self.k_proj = nn.Linear(C, H * N, bias=False)
            self.v_proj = nn.Linear(C, H * N, bias=False)
            self.g_proj = nn.Linear(C, H * N, bias=False)
            self.o_proj = nn.Linear(H * N, C, bias=False)
            for p in (self.q_proj, self.k_proj, self.v_proj, self.g_proj):
                p.weight.data.uniform_(-bound, bound)
            self.o_proj.weight.data.zero_()

    def forward(self, x: torch.Tensor, yarn) -> torch.Tensor:
        return fused_attn(x, self.q_proj, self.k_proj, self.v_proj, self.g_proj, self.o_proj, yarn,
                          self.num_heads, self.head_dim, save_o=self.save_o)
