"""Helpers shared by the GPU tests: call libmea entry points through the C ABI
and check the device status word after every call."""
import ctypes

import torch

from memory_efficient_attn_layer_b200 import _lib

DEV = torch.device("cuda", 0)


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def status():
    s = _lib.status_buffer(DEV)
    s.zero_()
    return s


def call(name, *args, status_buf=None):
    """Call libmea function `name`, raise on a non-zero code, then synchronise
    and raise if a bounded device wait gave up."""
    L = _lib.lib()
    _lib.check(getattr(L, name)(*args))
    torch.cuda.synchronize()
    if status_buf is not None:
        v = int(status_buf.item())
        assert v == 0, f"{name}: device wait timed out, status=0x{v:08x}"


def dims(B, T, C, H, N, T_max=None, eps=1e-6):
    return ctypes.byref(_lib.MeaBlockDims(B, T, C, H, N, T_max or T, eps))


def bf16(t):
    return t.to(device=DEV, dtype=torch.bfloat16).contiguous()


def maxrel(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def cos(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-300))
