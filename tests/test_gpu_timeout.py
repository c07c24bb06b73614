"""Device-side failure detection: a bounded wait that runs out is reported.

Every kernel of the library waits on mbarriers with a wall-clock limit; a wait
that gives up records (kernel id, wait site) in a device status word and the
kernel returns early.  mea_selftest_wait runs that same wait on a barrier that
nobody arrives on, with a 2 ms limit, so these tests see a real device timeout
without a fault or a hang (the wait always ends by its limit, and nothing else
is in flight in that kernel).  They check that the C ABI reports it, that the
default Python path raises MeaError(MEA_ERR_DEVICE_TIMEOUT) at the next call
without any per-call synchronisation, and that the calls after it run clean.
"""
import ctypes

import pytest
import torch

from memory_efficient_attn_layer_b200 import _lib

LIMIT_NS = 2_000_000  # 2 ms


def test_selftest_rejects_bad_arguments():
    L = _lib.lib()
    assert L.mea_selftest_wait(None, LIMIT_NS, 0, None) == 1
    assert L.mea_selftest_wait(ctypes.c_void_p(0x10000), 0, 0, None) == 1
    assert L.mea_selftest_wait(ctypes.c_void_p(0x10000), 2_000_000_000, 0, None) == 1
    assert b"limit_ns" in L.mea_last_error_string()


@pytest.mark.gpu
def test_c_abi_reports_a_wait_that_runs_out():
    from gpu_util import DEV, P, stream

    L = _lib.lib()
    s = torch.zeros(1, dtype=torch.int32, device=DEV)
    # the barrier completes: no error recorded
    _lib.check(L.mea_selftest_wait(P(s), LIMIT_NS, 1, stream()))
    out = ctypes.c_int(-1)
    assert L.mea_read_status(P(s), ctypes.byref(out), stream()) == 0 and out.value == 0
    # nobody arrives: the wait gives up after 2 ms and records kernel 9, site 1
    _lib.check(L.mea_selftest_wait(P(s), LIMIT_NS, 0, stream()))
    rc = L.mea_read_status(P(s), ctypes.byref(out), stream())
    assert rc == _lib.MEA_ERR_DEVICE_TIMEOUT
    assert out.value & 0xFF == 0x5A and (out.value >> 8) & 0xFF == 9 and (out.value >> 16) == 1
    assert b"kernel 9, site 1" in L.mea_last_error_string()
    # the context is still usable: the next wait completes and reports nothing
    s.zero_()
    _lib.check(L.mea_selftest_wait(P(s), LIMIT_NS, 1, stream()))
    assert L.mea_read_status(P(s), ctypes.byref(out), stream()) == 0 and out.value == 0


def _small_block_inputs():
    from gpu_util import DEV
    from oracle.eager import make_inputs

    H, N = 4, 32
    inp = make_inputs(1, 256, 128, H, N, seed=5)
    leaves = [inp[k].to(device=DEV, dtype=torch.bfloat16).requires_grad_(True)
              for k in ("x", "wq", "wk", "wv", "wg", "wo", "f1", "f2")]
    return inp, leaves, H, N


@pytest.mark.gpu
def test_default_path_raises_at_the_next_call_and_then_runs_clean():
    from gpu_util import DEV, P, stream
    from memory_efficient_attn_layer_b200 import FusedAttentionFunction, MeaError
    from oracle.eager import GRAD_NAMES, block_fwd_bwd, cos_sim, max_rel

    inp, leaves, H, N = _small_block_inputs()
    L = _lib.lib()
    # A timeout recorded in the library's own status word, followed by the same
    # asynchronous host copy every block call queues.
    word = _lib.status_buffer(DEV)
    word.zero_()
    _lib.check(L.mea_selftest_wait(P(word), LIMIT_NS, 0, stream()))
    _lib.note_status(DEV)
    torch.cuda.synchronize()  # lets the copy land; the library itself never waits for it
    with pytest.raises(MeaError) as err:
        FusedAttentionFunction.apply(*leaves, H, N, 1e-6)
    assert err.value.code == _lib.MEA_ERR_DEVICE_TIMEOUT
    assert "kernel 9, site 1" in str(err.value)
    # reported once, then cleared: the next call runs and matches the oracle
    y = FusedAttentionFunction.apply(*leaves, H, N, 1e-6)
    y.backward(inp["dy"].to(device=DEV, dtype=torch.bfloat16))
    _lib.check_device_status(DEV)
    want = block_fwd_bwd(inp, H, N)
    assert max_rel(y.detach().float().cpu(), want["y"]) < 2e-2
    for name, leaf in zip(GRAD_NAMES, leaves):
        assert cos_sim(leaf.grad.float().cpu(), want[name]) > 0.999, name


@pytest.mark.gpu
def test_check_device_status_reports_the_last_call():
    from gpu_util import DEV, P, stream
    from memory_efficient_attn_layer_b200 import MeaError

    L = _lib.lib()
    word = _lib.status_buffer(DEV)
    word.zero_()
    _lib.check(L.mea_selftest_wait(P(word), LIMIT_NS, 0, stream()))
    _lib.note_status(DEV)
    with pytest.raises(MeaError) as err:
        _lib.check_device_status(DEV)  # waits for the copy itself
    assert err.value.code == _lib.MEA_ERR_DEVICE_TIMEOUT
    _lib.check_device_status(DEV)  # cleared once reported
    assert int(word.item()) == 0
