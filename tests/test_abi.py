"""CPU: the C ABI library loads, exports every symbol include/mea.h declares,
and rejects bad arguments before touching a GPU."""
import ctypes

import pytest
import torch

from memory_efficient_attn_layer_b200 import _lib


@pytest.fixture(scope="module")
def L():
    return _lib.lib()


def test_exports_every_header_symbol(L):
    names = _lib.header_symbols()
    assert len(names) >= 16
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must mirror include/mea.h"


def test_version_and_error_string(L):
    assert L.mea_version() >= 100
    assert isinstance(L.mea_last_error_string(), bytes)


@pytest.mark.parametrize("dims,msg", [
    ((2, 100, 128, 4, 32, 256), b"multiple of 128"),
    ((2, 256, 128, 4, 48, 256), b"head dim"),
    ((2, 256, 96, 4, 32, 256), b"C=96"),
    ((2, 256, 128, 3, 32, 256), b"H*N"),
    ((2, 256, 128, 4, 32, 128), b"rotary tables"),
    ((0, 256, 128, 4, 32, 256), b"positive"),
])
def test_shape_validation(L, dims, msg):
    d = _lib.MeaBlockDims(*dims, 1e-6)
    assert L.mea_forward_workspace_size(ctypes.byref(d)) == 0
    assert L.mea_backward_workspace_size(ctypes.byref(d)) == 0
    rc = L.mea_block_forward(ctypes.byref(d), *([None] * 11), 0, None, None)
    assert rc in (1, 2)
    assert msg in L.mea_last_error_string()


def test_workspace_too_small_is_rejected(L):
    d = _lib.MeaBlockDims(2, 256, 128, 4, 32, 256, 1e-6)
    need = L.mea_forward_workspace_size(ctypes.byref(d))
    assert need > 0
    rc = L.mea_block_forward(ctypes.byref(d), *([None] * 10), ctypes.c_void_p(16), need - 1, None, None)
    assert rc == 7 and b"workspace" in L.mea_last_error_string()


def test_workspace_sizes_scale_with_batch(L):
    a = _lib.MeaBlockDims(1, 2048, 512, 8, 64, 2048, 1e-6)
    b = _lib.MeaBlockDims(2, 2048, 512, 8, 64, 2048, 1e-6)
    fa, fb = (L.mea_forward_workspace_size(ctypes.byref(x)) for x in (a, b))
    ba, bb = (L.mea_backward_workspace_size(ctypes.byref(x)) for x in (a, b))
    fixed = 5 * 512 * 512 * 4  # fp32 weight-gradient accumulators do not grow with B
    assert 1.9 < fb / fa < 2.1 and 1.9 < (bb - fixed) / (ba - fixed) < 2.1


def test_cpu_tensors_raise():
    from memory_efficient_attn_layer_b200 import FusedAttentionFunction
    x = torch.zeros(1, 128, 128, dtype=torch.bfloat16)
    w = torch.zeros(128, 128, dtype=torch.bfloat16)
    f = torch.zeros(128, 32, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        FusedAttentionFunction.apply(x, w, w, w, w, w, f, f, 4, 32, 1e-6)


def _fake(i):
    return ctypes.c_void_p(0x100000 * (i + 1))  # aligned stand-ins: the calls below never reach the device


@pytest.mark.parametrize("slot,bad,text", [
    (12, 0x7000002, b"weight-gradient output 0"),   # dwq only 2-byte aligned
    (16, 0x7000004, b"weight-gradient output 4"),   # dwo only 4-byte aligned
    (1, 0x7000008, b"tensor argument 0"),           # x only 8-byte aligned
    (11, 0x7000008, b"tensor argument 10"),         # dx only 8-byte aligned
])
def test_block_backward_rejects_misaligned_buffers_before_device_work(L, slot, bad, text):
    d = _lib.MeaBlockDims(2, 256, 128, 4, 32, 256, 1e-6)
    need = L.mea_backward_workspace_size(ctypes.byref(d))
    # d, x, wq, wk, wv, wg, wo, f1, f2, lse2, dy, dx, dwq, dwk, dwv, dwg, dwo, df1, df2, dw32, ws
    args = [ctypes.byref(d)] + [_fake(i) for i in range(20)]
    args[17] = args[18] = args[19] = None
    args[slot] = ctypes.c_void_p(bad)
    rc = L.mea_block_backward_ex(*args, need, None, None, None, None)
    assert rc == 3, L.mea_last_error_string()
    assert text in L.mea_last_error_string()


def test_block_forward_rejects_misaligned_output_before_device_work(L):
    d = _lib.MeaBlockDims(2, 256, 128, 4, 32, 256, 1e-6)
    need = L.mea_forward_workspace_size(ctypes.byref(d))
    args = [ctypes.byref(d)] + [_fake(i) for i in range(11)]
    args[9] = ctypes.c_void_p(0x7000002)  # y
    rc = L.mea_block_forward(*args, need, None, None)
    assert rc == 3 and b"tensor argument 8" in L.mea_last_error_string()


def test_gemm_e4m3_rejects_bad_arguments_before_device_work(L):
    a, b, o = (ctypes.c_void_p(0x100000 * i) for i in (1, 2, 3))
    assert L.mea_gemm_e4m3(256, 256, 192, a, 192, b, 192, o, 256, 0, None, None) == 2  # K % 128
    assert b"multiples" in L.mea_last_error_string()
    assert L.mea_gemm_e4m3(256, 256, 256, ctypes.c_void_p(0x100008), 256, b, 256, o, 256, 0, None, None) == 3
    assert L.mea_gemm_e4m3(256, 256, 256, None, 256, b, 256, o, 256, 0, None, None) == 1
