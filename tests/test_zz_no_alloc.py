"""mea_attention_backward_noalloc: the attention backward for callers that
cannot allocate device memory.

Some callers of this library cannot call cudaMalloc: a plugin whose execute
callback runs inside a host runtime that forbids allocation there (or cannot
afford the device synchronisation it may cause), or code that is handed only
its input and output buffers and no allocator.  For them the fp32 dQ
accumulator that mea_attention_backward takes from its caller lives in a fixed
16 MiB array inside libmea.so.  These tests check that entry point through the
C ABI against the ordinary one, on two calls in a row (the shared array must be
cleared by each call), and that oversized problems are rejected.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from memory_efficient_attn_layer_b200 import _lib

LIMIT = 4 * 1024 * 1024  # fp32 elements in the built-in accumulator


def test_noalloc_rejects_problems_above_the_limit():
    L = _lib.lib()
    # B*H*T*N = 8*8*2048*64 = 8,388,608 > 4,194,304: rejected before any device work
    rc = L.mea_attention_backward_noalloc(8, 8, 2048, 64, *([None] * 9), 512, None, None)
    assert rc == 2
    assert b"exceeds the built-in limit" in L.mea_last_error_string()


# Every argument is checked before the entry point queues any device work (a
# rejected call leaves the caller's stream untouched), so these run without a
# GPU.  Fake but aligned device addresses stand in for the tensors.
_FAKE = [0x10000 * (i + 1) for i in range(9)]  # q, k, v, dO, lse2, delta, dq, dk, dv


@pytest.mark.parametrize("case,dims,override,code,text", [
    ("null dq", (1, 2, 256, 64), {6: None}, 1, b"dq is NULL"),
    ("zero batch", (0, 2, 256, 64), {}, 1, b"dims must be positive"),
    ("T not a multiple of 128", (1, 2, 100, 64), {}, 2, b"multiple of 128"),
    ("head dim 48", (1, 2, 256, 48), {}, 2, b"head dim 48"),
    ("dq 2-byte aligned", (1, 2, 256, 64), {6: 0x70002}, 3, b"dq must be 8-byte aligned"),
    ("dk 8-byte aligned", (1, 2, 256, 64), {7: 0x80008}, 3, b"dk/dv must be 16-byte aligned"),
    ("null q", (1, 2, 256, 64), {0: None}, 1, b"NULL tensor pointer"),
])
def test_noalloc_rejects_bad_arguments_before_device_work(case, dims, override, code, text):
    L = _lib.lib()
    ptrs = list(_FAKE)
    for i, v in override.items():
        ptrs[i] = v
    B, H, T, N = dims
    rc = L.mea_attention_backward_noalloc(B, H, T, N, *ptrs, H * N, None, None)
    assert rc == code, (case, rc, L.mea_last_error_string())
    assert text in L.mea_last_error_string(), case


@pytest.mark.gpu
@pytest.mark.parametrize("N", [32, 64, 128])
def test_noalloc_matches_allocating_entry_point_twice(N):
    from gpu_util import DEV, P, call, cos, maxrel, status, stream

    B, H, T = 2, 2, 384
    assert B * H * T * N <= LIMIT
    g = torch.Generator(device=DEV).manual_seed(123)

    def unit_rms(t):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True))

    q = unit_rms(torch.randn(B, H, T, N, device=DEV, generator=g)).bfloat16().contiguous()
    k = unit_rms(torch.randn(B, H, T, N, device=DEV, generator=g)).bfloat16().contiguous()
    v = torch.randn(B, H, T, N, device=DEV, generator=g).bfloat16().contiguous()
    dO = torch.randn(B, H, T, N, device=DEV, generator=g).bfloat16().contiguous()
    ones = torch.ones_like(q)
    gated = torch.empty(B, T, H * N, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(B, H, T, device=DEV)
    o = torch.empty_like(q)
    s = status()
    call("mea_attention_forward", B, H, T, N, P(q), P(k), P(v), P(ones), P(gated), P(lse), P(o), P(s), stream(),
         status_buf=s)
    delta = (dO.float() * o.float()).sum(-1).contiguous()

    # the ordinary entry point, with a caller-allocated fp32 dq accumulator
    dq_acc = torch.zeros(B, H, T, N, device=DEV)
    dk_ref = torch.empty_like(q)
    dv_ref = torch.empty(B, T, H, N, dtype=torch.bfloat16, device=DEV)
    call("mea_attention_backward", B, H, T, N, P(q), P(k), P(v), P(dO), P(lse), P(delta), P(dq_acc), P(dk_ref),
         P(dv_ref), H * N, P(s), stream(), status_buf=s)

    for _ in range(2):  # the built-in accumulator must be cleared on every call
        dq = torch.full_like(q, float("nan"))
        dk = torch.full_like(q, float("nan"))
        dv = torch.full((B, T, H, N), float("nan"), dtype=torch.bfloat16, device=DEV)
        call("mea_attention_backward_noalloc", B, H, T, N, P(q), P(k), P(v), P(dO), P(lse), P(delta), P(dq), P(dk),
             P(dv), H * N, P(s), stream(), status_buf=s)
        for name, got, want in (("dq", dq, dq_acc), ("dk", dk, dk_ref), ("dv", dv, dv_ref)):
            assert torch.isfinite(got.float()).all(), name
            assert maxrel(got.float(), want.float()) < 2e-2, name
            assert cos(got.float(), want.float()) > 0.999, name
