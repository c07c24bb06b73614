"""CPU oracle for the sharded AdamW step -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/`` may import it.
The CUDA path (``mea_adamw_step`` in libmea.so, driven by
``memory_efficient_attn_layer_b200.optim.ShardedAdamW``) never calls it.

The reference project has no optimizer: its module (README.md:6-68) is
trained by whatever optimizer its caller picks.  The step restated here is
Adam (Kingma & Ba, 2015) with decoupled weight decay (Loshchilov & Hutter,
2019) in the operation order torch.optim.AdamW uses, computed in numpy fp32
with the scalar schedule in fp64:

    w  <- w * (1 - lr*wd)
    m  <- m + (1 - b1) * (g - m)
    v  <- v * b2 + (1 - b2) * g*g
    w  <- w - (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps),   bc_i = 1 - b_i**step

with g = grad * grad_scale.  ``tests/test_optim_cpu.py`` pins this restatement
against torch.optim.AdamW itself on CPU over several steps.
"""
from __future__ import annotations

import math

import numpy as np


def adamw_step(master: np.ndarray, exp_avg: np.ndarray, exp_avg_sq: np.ndarray, grad: np.ndarray, *, lr: float,
               beta1: float, beta2: float, eps: float, weight_decay: float, step: int,
               grad_scale: float = 1.0) -> np.ndarray:
    """One AdamW step in place on fp32 arrays; returns the bf16-rounded new
    weights as a float32 array (round to nearest even, the kernel's cast)."""
    f = np.float32
    g = grad.astype(f) * f(grad_scale)
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    master *= f(1.0 - lr * weight_decay)
    exp_avg += f(1.0 - beta1) * (g - exp_avg)
    exp_avg_sq *= f(beta2)
    exp_avg_sq += f(1.0 - beta2) * (g * g)
    denom = np.sqrt(exp_avg_sq) / f(math.sqrt(bc2)) + f(eps)
    master -= f(lr / bc1) * (exp_avg / denom)
    return to_bf16(master)


def to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest, ties to even) -> fp32, elementwise."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return rounded.view(np.float32)
