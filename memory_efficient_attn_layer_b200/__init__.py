"""B200-native (sm_100a) gated causal attention block.

Drop-in for xTimeCrystal/memory_efficient_attn_layer: ``fused_attn``,
``FusedAttentionFunction`` and ``CausalSoftmaxAttention`` keep the reference's
names and call surface; the work runs in hand-written tcgen05/TMA kernels in
``libmea.so`` (C ABI in ``include/mea.h``).
"""
from ._lib import MeaError, check_device_status
from .dp import allreduce_grads, overlap_grad_allreduce
from .fused_attn import FusedAttentionFunction, fused_attn
from .module import CausalSoftmaxAttention, Yarn
from .optim import ShardedAdamW

__all__ = ["fused_attn", "FusedAttentionFunction", "CausalSoftmaxAttention", "Yarn", "allreduce_grads",
           "overlap_grad_allreduce", "ShardedAdamW", "MeaError", "check_device_status"]
